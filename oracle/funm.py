"""CPU (numpy) restatement of the reference's matrix-function primitive:
m-step Lanczos quadrature for f(A) v and v^T f(A) v.

TEST INFRASTRUCTURE ONLY: imported by tests/ to check results; the product path
never imports it.  The reference's CUDA path links LAPACK and cannot run here;
the restatement is pinned (tests/test_oracle_funm.py) against the dense
ground truth U f(Lambda) U^T v that the reference's own tests use
(tests/test_funm.py:48-62 of the reference), exact when the Krylov space is
exhausted.

Follows (reference file:line):
  lanczos_extend_funm (CGS + conditional DGKS, stop at an invariant
    subspace) ................................ src/matrix_function.cuh:82-126
  lanczos_build_basis ........................ src/matrix_function.cuh:137-170
  quadratic form / apply ..................... src/matrix_function.cuh:187-240
  apply_scalar_func (domain rules, codes) .... src/matrix_function.cuh:251-274
  compute_funm_apply / _qform return codes ... python/gpu_eigsh/_cuda_funm.cu:40-251
"""
from __future__ import annotations

import numpy as np

EPS23 = np.finfo(np.float64).eps ** (2.0 / 3.0)
SAFE_MIN = np.finfo(np.float64).tiny


def _breakdown_tol(alpha, beta, j):
    est = 0.0
    for i in range(j + 1):
        rs = abs(alpha[i]) + (abs(beta[i]) if i > 0 else 0.0) + (abs(beta[i + 1]) if i < j else 0.0)
        est = max(est, rs)
    return EPS23 * max(est, SAFE_MIN)


def lanczos_basis(A, v, m):
    """(V n x m_actual, alpha, beta (m_actual + 1), ||v||).  Classical
    Gram-Schmidt, then DGKS (src/lanczos_ops.cuh:147-192): when
    ||r|| <= ||w|| / sqrt(2), up to two correction passes, each accepted when
    it keeps more than 1/sqrt(2) of the norm; two failed passes mean an
    invariant subspace (||r|| = 0)."""
    n = v.shape[0]
    vnorm = float(np.linalg.norm(v))
    if vnorm == 0.0:
        return np.zeros((n, 0)), np.zeros(0), np.zeros(1), 0.0
    V = np.zeros((n, m))
    alpha = np.zeros(m)
    beta = np.zeros(m + 1)
    V[:, 0] = v / vnorm
    for j in range(m):
        w = A @ V[:, j]
        wn = np.linalg.norm(w)
        h = V[:, :j + 1].T @ w
        r = w - V[:, :j + 1] @ h
        alpha[j] = h[j]
        rn = np.linalg.norm(r)
        eta = 1.0 / np.sqrt(2.0)
        if not rn > eta * wn:
            for p in range(2):
                s = V[:, :j + 1].T @ r
                r = r - V[:, :j + 1] @ s
                alpha[j] += s[j]
                rn_new = np.linalg.norm(r)
                if rn_new > eta * rn:
                    rn = rn_new
                    break
                if p == 1:
                    rn = 0.0
                    break
                rn = rn_new
        if rn < _breakdown_tol(alpha, beta, j):
            beta[j + 1] = 0.0
            return V[:, :j + 1], alpha[:j + 1], beta[:j + 2], vnorm
        if j + 1 < m:
            beta[j + 1] = rn
            V[:, j + 1] = r / rn
        else:
            beta[m] = rn
    return V, alpha, beta, vnorm


def scalar_func(name, theta):
    """(f(theta), status) with the reference's domain rules."""
    if name == "log":
        return (np.log(theta), 0) if np.all(theta > 0) else (None, -2)
    if name == "exp":
        return np.exp(theta), 0
    if name == "sqrt":
        return (np.sqrt(theta), 0) if np.all(theta >= 0) else (None, -2)
    if name == "inv":
        return (1.0 / theta, 0) if np.all(theta != 0) else (None, -2)
    return None, -1


def funm(A, v, m, func, mode):
    """mode 'apply' -> (y, status_or_depth); mode 'qform' -> (value, ...)."""
    if func not in ("log", "exp", "sqrt", "inv"):
        return None, -1
    V, alpha, beta, vnorm = lanczos_basis(A, np.asarray(v, dtype=np.float64), int(m))
    ma = alpha.shape[0]
    if ma == 0:
        return (np.zeros(A.shape[0]) if mode == "apply" else 0.0), -3
    T = np.diag(alpha) + np.diag(beta[1:ma], 1) + np.diag(beta[1:ma], -1)
    theta, S = np.linalg.eigh(T)
    f, st = scalar_func(func, theta)
    if st:
        return None, st
    if mode == "qform":
        return float(vnorm * vnorm * np.sum(S[0, :] ** 2 * f)), ma
    q = S @ (f * S[0, :])
    return vnorm * (V @ q), ma


def dense_funm_apply(A, v, func):
    """U f(Lambda) U^T v by the dense eigendecomposition (the reference's ground truth)."""
    w, U = np.linalg.eigh(A.toarray())
    f = {"log": np.log, "exp": np.exp, "sqrt": np.sqrt, "inv": lambda x: 1.0 / x}[func](w)
    return U @ (f * (U.T @ v))


def spd_laplacian(n, eps_shift=1e-2, nn=10, seed=42):
    """The reference's funm test matrix (tests/test_funm.py:27-45): kNN graph
    Laplacian of 5-D Gaussian points plus eps I."""
    import scipy.sparse as sp
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((n, 5))
    d, ix = cKDTree(pts).query(pts, k=nn + 1)
    rows = np.repeat(np.arange(n), nn)
    W = sp.csr_matrix((np.exp(-(d[:, 1:] ** 2) / 4.0).ravel(), (rows, ix[:, 1:].ravel())), shape=(n, n))
    W = W.maximum(W.T)
    deg = np.asarray(W.sum(axis=1)).ravel()
    L = sp.diags(deg) - W + sp.diags(np.full(n, eps_shift))
    L = L.tocsr()
    L.sort_indices()
    return L
