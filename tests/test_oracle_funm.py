"""Pins of the matrix-function oracle (oracle/funm.py) on CPU against the
dense ground truth the reference's own tests use (tests/test_funm.py of the
reference): U f(Lambda) U^T v, with the reference's thresholds, and exactness
once the Krylov space is exhausted."""
import numpy as np
import pytest

from oracle import funm as OF

# (n, m, func, threshold) as the reference's test table
CASES = [(100, 80, "log", 1e-8), (100, 80, "exp", 1e-8), (100, 80, "sqrt", 1e-8), (100, 80, "inv", 1e-6),
         (500, 50, "log", 1e-3), (500, 50, "exp", 1e-3), (500, 50, "sqrt", 1e-3), (500, 50, "inv", 1e-1)]


@pytest.mark.parametrize("n,m,func,thr", CASES)
def test_oracle_matches_dense_ground_truth(n, m, func, thr):
    L = OF.spd_laplacian(n, seed=7)
    v = np.random.default_rng(0).standard_normal(n)
    y, ma = OF.funm(L, v, m, func, "apply")
    q, _ = OF.funm(L, v, m, func, "qform")
    ref = OF.dense_funm_apply(L, v, func)
    assert ma == m
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < thr
    assert abs(q - v @ ref) / abs(v @ ref) < thr


def test_exhausted_krylov_space_is_exact():
    """A matrix with 6 distinct eigenvalues: the basis stops at depth 6
    (invariant subspace) and the quadrature is exact."""
    import scipy.sparse as sp

    d = np.repeat([1.0, 2.0, 3.5, 4.0, 7.0, 9.0], 20)
    A = sp.diags(d).tocsr()
    v = np.random.default_rng(1).standard_normal(d.size)
    y, ma = OF.funm(A, v, 30, "log", "apply")
    assert ma == 6
    np.testing.assert_allclose(y, np.log(d) * v, rtol=1e-12, atol=1e-12)


def test_status_codes():
    import scipy.sparse as sp

    A = sp.diags(np.linspace(-1.0, 2.0, 50)).tocsr()
    v = np.ones(50)
    assert OF.funm(A, v, 10, "log", "apply")[1] == -2
    assert OF.funm(A, v, 10, "exp", "apply")[1] == 10
    assert OF.funm(A, np.zeros(50), 10, "exp", "qform")[1] == -3
    assert OF.funm(A, v, 10, "cosh", "apply")[1] == -1
