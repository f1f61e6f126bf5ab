"""Shared parity assertions for eigenvalue tests."""
import numpy as np


def eig_rel_err(w, ref, anorm):
    """Max relative error; eigenvalues below 1e-8*||A|| are compared absolutely
    against 1e-12*||A|| instead (relative error of a zero eigenvalue is
    meaningless; the reference's own test skips lambda_0)."""
    w = np.asarray(w, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    tiny = np.abs(ref) < 1e-8 * anorm
    err = np.zeros_like(ref)
    err[~tiny] = np.abs(w[~tiny] - ref[~tiny]) / np.abs(ref[~tiny])
    # scaled so that 1e-12*||A|| absolute maps to 1e-10
    err[tiny] = np.abs(w[tiny] - ref[tiny]) / (1e-2 * anorm)
    return float(err.max()) if err.size else 0.0


def anorm1(A):
    return float(abs(A).sum(axis=1).max())
