"""GPU parity of the matrix-function primitive (gpu_eigsh.funm_apply /
funm_qform, lg_eigsh_plan_funm, compute_funm_*).

Checked against the oracle (oracle/funm.py: the reference's Lanczos quadrature
restated, pinned to the dense ground truth by tests/test_oracle_funm.py) at
1e-10 relative (the CUDA basis uses CGS2, the reference CGS + conditional
DGKS: the tridiagonals agree to rounding), against the dense ground truth with
the reference's thresholds, and for the reference's status codes.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [(100, 80, "log", 1e-8), (100, 80, "exp", 1e-8), (100, 80, "sqrt", 1e-8), (100, 80, "inv", 1e-6),
         (500, 50, "log", 1e-3), (500, 50, "exp", 1e-3), (500, 50, "sqrt", 1e-3), (500, 50, "inv", 1e-1),
         (1000, 80, "log", 1e-4), (1000, 80, "exp", 1e-4), (1000, 80, "sqrt", 1e-4), (1000, 80, "inv", 1e-1)]


@pytest.fixture(scope="module")
def ge():
    import gpu_eigsh

    return gpu_eigsh


@pytest.mark.parametrize("n,m,func,thr", CASES)
def test_funm_matches_oracle_and_dense(ge, n, m, func, thr):
    from oracle import funm as OF

    L = OF.spd_laplacian(n, seed=7)
    v = np.random.default_rng(0).standard_normal(n)
    y, ma = ge.funm_apply(L, v, m=m, func=func)
    q, mq = ge.funm_qform(L, v, m=m, func=func)
    yo, mo = OF.funm(L, v, m, func, "apply")
    qo, _ = OF.funm(L, v, m, func, "qform")
    assert ma == mo == mq
    assert np.linalg.norm(y - yo) / np.linalg.norm(yo) < 1e-10
    assert abs(q - qo) / abs(qo) < 1e-10
    ref = OF.dense_funm_apply(L, v, func)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < thr
    assert abs(q - v @ ref) / abs(v @ ref) < thr


def test_funm_exhausted_krylov_space(ge):
    import scipy.sparse as sp

    d = np.repeat([1.0, 2.0, 3.5, 4.0, 7.0, 9.0], 20)
    A = sp.diags(d).tocsr()
    v = np.random.default_rng(1).standard_normal(d.size)
    y, ma = ge.funm_apply(A, v, m=30, func="log")
    assert ma == 6
    np.testing.assert_allclose(y, np.log(d) * v, rtol=1e-11, atol=1e-11)


def test_funm_status_codes(ge):
    import scipy.sparse as sp

    A = sp.diags(np.linspace(-1.0, 2.0, 50)).tocsr()
    with pytest.raises(RuntimeError, match="invalid eigenvalue for func"):
        ge.funm_apply(A, np.ones(50), m=10, func="log")
    with pytest.raises(RuntimeError, match="zero input vector"):
        ge.funm_qform(A, np.zeros(50), m=10, func="exp")
    with pytest.raises(RuntimeError, match="unknown func"):
        ge.funm_apply(A, np.ones(50), m=10, func="cosh")
    q, ma = ge.funm_qform(A, np.ones(50), m=10, func="exp")
    assert ma == 10 and np.isfinite(q)


def test_reference_abi_funm(ge):
    """compute_funm_apply / _qform / _debug with the reference's signatures and
    return codes; the debug basis is orthonormal and V^T A V = T."""
    from gpu_eigsh import _native
    from oracle import funm as OF

    L = OF.spd_laplacian(300, seed=3)
    n, m = 300, 40
    v = np.random.default_rng(2).standard_normal(n)
    PI, PD = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)
    ip = np.ascontiguousarray(L.indptr, dtype=np.int32)
    ix = np.ascontiguousarray(L.indices, dtype=np.int32)
    dv = np.ascontiguousarray(L.data, dtype=np.float64)
    args = (n, L.nnz, ip.ctypes.data_as(PI), ix.ctypes.data_as(PI), dv.ctypes.data_as(PD), v.ctypes.data_as(PD), m)
    y = np.zeros(n)
    assert _native.lib.compute_funm_apply(*args, b"sqrt", y.ctypes.data_as(PD)) == m
    np.testing.assert_allclose(y, ge.funm_apply(L, v, m=m, func="sqrt")[0], rtol=0, atol=0)
    val = ctypes.c_double()
    assert _native.lib.compute_funm_qform(*args, b"log", ctypes.byref(val)) == m
    assert abs(val.value - OF.funm(L, v, m, "log", "qform")[0]) < 1e-10 * abs(val.value)
    assert _native.lib.compute_funm_qform(*args, b"nope", ctypes.byref(val)) == -1
    V = np.zeros(n * m)
    a = np.zeros(m)
    b = np.zeros(m + 1)
    assert _native.lib.compute_funm_debug(*args, V.ctypes.data_as(PD), a.ctypes.data_as(PD),
                                          b.ctypes.data_as(PD)) == m
    V = V.reshape(m, n).T
    np.testing.assert_allclose(V.T @ V, np.eye(m), atol=1e-12)
    T = np.diag(a) + np.diag(b[1:m], 1) + np.diag(b[1:m], -1)
    np.testing.assert_allclose(V.T @ (L @ V), T, atol=1e-10)
    Vo, ao, bo, _ = OF.lanczos_basis(L, v, m)
    np.testing.assert_allclose(a, ao, rtol=1e-11)
    np.testing.assert_allclose(b, bo, rtol=1e-11)
