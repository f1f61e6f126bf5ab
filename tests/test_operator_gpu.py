"""GPU parity of eigsh on matrix-free operators (the reference's
FunctionOperator, src/matvec_operator.cuh:149-163, reached through
lg_eigsh_plan_create_op).

The kNN Laplacian is handed to the solver only as a function y = A x, in the
three forms the C ABI takes: a scipy LinearOperator on the host (LG_OP_HOST),
a torch function on the solver's CUDA stream (LG_OP_STREAM), and a raw
function of two device pointers (LG_OP_DEVICE, the reference's contract).
Eigenvalues match scipy ARPACK to 1e-10 relative, every Ritz pair satisfies
||A v - lambda v|| <= tol * ||A||, as for CSR plans.
"""
import numpy as np
import pytest

from _parity import anorm1, eig_rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def knn():
    from gpu_eigsh import synthetic as syn

    L, _ = syn.knn_laplacian(20000, k=10, seed=12)
    v0 = np.random.default_rng(8).standard_normal(L.shape[0])
    return L, v0


@pytest.fixture(scope="module")
def arpack(knn):
    from oracle.irlm import arpack_eigsh

    L, v0 = knn
    return arpack_eigsh(L, 10, which="LA", ncv=36, tol=1e-10, v0=v0)


def _check(L, w, V, ws):
    an = anorm1(L)
    assert eig_rel_err(w, ws, an) < 1e-10
    res = np.linalg.norm(L @ V - V * w, axis=0)
    assert res.max() <= 1e-10 * an
    np.testing.assert_allclose(V.T @ V, np.eye(V.shape[1]), atol=1e-9)


def test_linear_operator_on_host_vs_arpack(knn, arpack):
    import gpu_eigsh
    from scipy.sparse.linalg import LinearOperator

    L, v0 = knn
    calls = []

    def mv(x):
        calls.append(1)
        return L @ x

    op = LinearOperator(L.shape, matvec=mv, dtype=np.float64)
    (w, V), info = gpu_eigsh.gpu_eigsh(op, k=10, which="LA", ncv=36, tol=1e-10, v0=v0, return_info=True)
    _check(L, w, V, arpack[0])
    # one product per Lanczos step
    assert len(calls) == info["steps"]


def test_cuda_operator_on_solver_stream_vs_arpack(knn, arpack):
    import torch

    import gpu_eigsh

    L, v0 = knn
    dev = torch.device("cuda")
    Lt = torch.sparse_csr_tensor(torch.from_numpy(L.indptr.astype(np.int64)),
                                 torch.from_numpy(L.indices.astype(np.int64)), torch.from_numpy(L.data),
                                 L.shape).to(dev)
    op = gpu_eigsh.CudaOperator(L.shape[0], lambda x: Lt @ x, device=dev)
    w, V = gpu_eigsh.gpu_eigsh(op, k=10, which="LA", ncv=36, tol=1e-10, v0=v0)
    _check(L, w, V, arpack[0])


def test_raw_device_callback_vs_arpack(knn, arpack):
    """LG_OP_DEVICE: a function of two device pointers (here the library's
    own CSR product of a second plan); the solver drains its stream before
    each call and the device after it."""
    import gpu_eigsh
    from gpu_eigsh.operators import raw_device_callback

    L, v0 = knn
    with gpu_eigsh.EigshPlan(L, max_ncv=8) as csr:
        cb = raw_device_callback(lambda x, y, n: csr.matvec_device(x, y))
        with gpu_eigsh.EigshPlan(L.shape[0], max_ncv=40, callback=cb) as plan:
            w, V = plan.solve(k=10, which="LA", ncv=36, tol=1e-10, v0=v0)
    _check(L, w, V, arpack[0])


@pytest.mark.parametrize("which", ["SA", "LM"])
def test_operator_which_vs_arpack(knn, which):
    import gpu_eigsh
    from oracle.irlm import arpack_eigsh
    from scipy.sparse.linalg import aslinearoperator

    L, v0 = knn
    Ls = L[:4000, :4000].tocsr()
    v = v0[:4000]
    w, V = gpu_eigsh.gpu_eigsh(aslinearoperator(Ls), k=6, which=which, ncv=30, tol=1e-10, v0=v)
    ws, _ = arpack_eigsh(Ls, 6, which=which, ncv=30, tol=1e-10, v0=v)
    assert eig_rel_err(w, ws, anorm1(Ls)) < 1e-10


def test_operator_factorization_equals_csr_inline(knn):
    """Same Lanczos tridiagonal as a CSR plan with in-step CGS2 (the steps an
    operator plan runs), to rounding."""
    import gpu_eigsh
    from scipy.sparse.linalg import aslinearoperator

    L, v0 = knn
    with gpu_eigsh.EigshPlan(L, max_ncv=64, cgs2_inline=True) as p:
        a0, b0 = p.factorize(v0, 50)
    with gpu_eigsh.EigshPlan(aslinearoperator(L), max_ncv=64) as p:
        a1, b1 = p.factorize(v0, 50)
    scale = np.abs(a0).max()
    assert np.max(np.abs(a0 - a1)) < 1e-12 * scale
    assert np.max(np.abs(b0 - b1)) < 1e-12 * scale


def test_operator_exception_is_raised(knn):
    """An exception inside the caller's matvec stops the solve (its product is
    NaN) and comes back from solve()."""
    import torch

    import gpu_eigsh

    L, v0 = knn
    n = L.shape[0]
    count = [0]

    def bad(x):
        count[0] += 1
        if count[0] == 5:
            raise KeyError("operator failed")
        return 2.0 * x

    op = gpu_eigsh.CudaOperator(n, bad, device=torch.device("cuda"))
    with pytest.raises(KeyError, match="operator failed"):
        gpu_eigsh.gpu_eigsh(op, k=4, which="LA", ncv=20, tol=1e-10, v0=v0)
