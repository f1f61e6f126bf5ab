"""GPU parity of the differentiable eigsh (forward + implicit-differentiation
backward, gpu_eigsh.differentiable / lg_eigsh_adjoint).

Checked against
  * the dense torch.linalg.eigh backward for eigenvalue losses (exact:
    Hellmann-Feynman), as the reference's tests/test_gradient.py does;
  * the oracle (oracle/adjoint.py: the reference's compute_adjoint_eigsh
    restated, pinned by tests/test_oracle_adjoint.py) on the SAME eigenpairs
    for eigenvector losses: the block CG on the GPU and the oracle's per-pair
    CG converge to the same deflated solutions, so the gradients agree to the
    CG tolerance (1e-12 relative here);
  * central finite differences for a single-eigenvector loss (k = 1).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    return torch


def _csr_tensor(torch, L, device="cuda", requires_grad=True):
    crow = torch.from_numpy(L.indptr.astype(np.int64)).to(device)
    col = torch.from_numpy(L.indices.astype(np.int64)).to(device)
    vals = torch.from_numpy(L.data.astype(np.float64)).to(device).requires_grad_(requires_grad)
    return torch.sparse_csr_tensor(crow, col, vals, L.shape), vals


def _pattern_rows(L):
    return np.repeat(np.arange(L.shape[0]), np.diff(L.indptr))


def test_eigenvalue_gradient_matches_dense_eigh(torch_cuda):
    torch = torch_cuda
    from gpu_eigsh import differentiable_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(100)
    k = 5
    Ld = torch.from_numpy(L.toarray()).requires_grad_(True)
    ev, _ = torch.linalg.eigh(Ld)
    ev[1:k].sum().backward()
    dense = Ld.grad.numpy()[_pattern_rows(L), L.indices]
    A, vals = _csr_tensor(torch, L)
    w, V = differentiable_eigsh(A, k=k, tol=1e-12, cg_tol=1e-10, cg_max_iters=500)
    np.testing.assert_allclose(w.detach().cpu().numpy(), ev[:k].detach().numpy(), rtol=0, atol=1e-12)
    w[1:].sum().backward()
    np.testing.assert_allclose(vals.grad.cpu().numpy(), dense, rtol=0, atol=1e-10)


def test_hellmann_feynman_single_eigenvalue(torch_cuda):
    torch = torch_cuda
    from gpu_eigsh import differentiable_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(200)
    A, vals = _csr_tensor(torch, L)
    w, V = differentiable_eigsh(A, k=3, tol=1e-12, cg_tol=1e-10)
    w[1].backward()
    x = V[:, 1].detach().cpu().numpy()
    hf = x[_pattern_rows(L)] * x[L.indices]
    np.testing.assert_allclose(vals.grad.cpu().numpy(), hf, rtol=0, atol=1e-13)


@pytest.mark.parametrize("n,k,seed", [(300, 5, 0), (2000, 20, 1), (500, 33, 2)])
def test_eigenvector_gradient_matches_oracle(torch_cuda, n, k, seed):
    """Random upstream gradients on eigenvalues and eigenvectors; the oracle
    runs the reference's per-pair deflated CG on the same eigenpairs."""
    torch = torch_cuda
    from gpu_eigsh import differentiable_eigsh
    from oracle import adjoint as OA

    L = OA.reference_test_laplacian(n, seed=seed)
    A, vals = _csr_tensor(torch, L)
    w, V = differentiable_eigsh(A, k=k, ncv=min(3 * k + 10, n - 1), tol=1e-12, cg_tol=1e-12, cg_max_iters=3000)
    rng = np.random.default_rng(seed)
    ge = rng.standard_normal(k)
    gv = rng.standard_normal((n, k))
    ((w * torch.from_numpy(ge).cuda()).sum() + (V * torch.from_numpy(gv).cuda()).sum()).backward()
    got = vals.grad.cpu().numpy()
    ref, iters = OA.adjoint_eigsh(L, w.detach().cpu().numpy(), V.detach().cpu().numpy(), g_evals=ge, g_evecs=gv,
                                  cg_max_iters=3000, cg_tol=1e-12)
    assert all(i > 0 for i in iters)
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 1e-8 * scale, np.abs(got - ref).max() / scale


def test_single_eigenvector_gradient_matches_finite_differences(torch_cuda):
    torch = torch_cuda
    from gpu_eigsh import differentiable_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(80, nn=6, seed=5)
    n = L.shape[0]
    u = torch.from_numpy(np.random.default_rng(1).standard_normal(n)).cuda()
    A, vals = _csr_tensor(torch, L)
    w, V = differentiable_eigsh(A, k=1, ncv=20, tol=1e-13, cg_tol=1e-13, cg_max_iters=5000)
    ((V[:, 0] * u).sum() ** 2).backward()
    grad = vals.grad.cpu().numpy()
    rows = _pattern_rows(L)
    pos = {(r, c): p for p, (r, c) in enumerate(zip(rows, L.indices))}
    un = u.cpu().numpy()

    def loss(M):
        _, VV = np.linalg.eigh(M)
        return float((un @ VV[:, 0]) ** 2)

    h = 1e-6
    rng = np.random.default_rng(3)
    for p in rng.choice(L.nnz, 25, replace=False):
        r, c = int(rows[p]), int(L.indices[p])
        E = np.zeros((n, n))
        E[r, c] += h
        if r != c:
            E[c, r] += h
        fd = (loss(L.toarray() + E) - loss(L.toarray() - E)) / (2 * h)
        an = grad[p] + (grad[pos[(c, r)]] if r != c else 0.0)
        assert abs(fd - an) <= 1e-6 * max(1.0, abs(fd)), (r, c, fd, an)


def test_shift_invert_forward_and_gradient(torch_cuda):
    torch = torch_cuda
    from gpu_eigsh import differentiable_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(500)
    A, vals = _csr_tensor(torch, L)
    w0, _ = differentiable_eigsh(A, k=6, tol=1e-12)
    A2, vals2 = _csr_tensor(torch, L)
    w1, V1 = differentiable_eigsh(A2, k=6, sigma=-0.05, tol=1e-12, cg_tol=1e-13, cg_max_iters=5000)
    np.testing.assert_allclose(w1.detach().cpu().numpy(), w0.detach().cpu().numpy(), rtol=0, atol=1e-10)
    w1[2].backward()
    x = V1[:, 2].detach().cpu().numpy()
    np.testing.assert_allclose(vals2.grad.cpu().numpy(), x[_pattern_rows(L)] * x[L.indices], rtol=0, atol=1e-12)


def test_cpu_values_and_reference_abi(torch_cuda):
    """Values on the CPU come back on the CPU; the reference-compatible host
    entry point compute_adjoint_eigsh gives the same gradient."""
    torch = torch_cuda
    from gpu_eigsh import _native, differentiable_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(400, seed=7)
    n, k = L.shape[0], 4
    A, vals = _csr_tensor(torch, L, device="cpu")
    w, V = differentiable_eigsh(A, k=k, tol=1e-12, cg_tol=1e-12)
    assert w.device.type == "cpu" and V.device.type == "cpu"
    gv = np.random.default_rng(4).standard_normal((n, k))
    (V * torch.from_numpy(gv)).sum().backward()
    assert vals.grad.device.type == "cpu"
    out = np.zeros(L.nnz)
    PI, PD = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)
    ip = np.ascontiguousarray(L.indptr, dtype=np.int32)
    ix = np.ascontiguousarray(L.indices, dtype=np.int32)
    dv = np.ascontiguousarray(L.data, dtype=np.float64)
    wn = np.ascontiguousarray(w.detach().numpy())
    Vn = np.ascontiguousarray(V.detach().numpy())
    rc = _native.lib.compute_adjoint_eigsh(n, L.nnz, ip.ctypes.data_as(PI), ix.ctypes.data_as(PI),
                                           dv.ctypes.data_as(PD), k, wn.ctypes.data_as(PD), Vn.ctypes.data_as(PD),
                                           None, gv.ctypes.data_as(PD), out.ctypes.data_as(PD), 500, 1e-12)
    assert rc == 0
    np.testing.assert_array_equal(out, vals.grad.numpy())   # same kernels, same order: bitwise


def test_adjoint_rejects_malformed_csr(torch_cuda):
    """A column index out of range is caught on the device before any kernel
    gathers through it."""
    torch = torch_cuda
    from gpu_eigsh import _native
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(50)
    n, k = L.shape[0], 2
    rp = torch.from_numpy(L.indptr.astype(np.int32)).cuda()
    ci = torch.from_numpy(L.indices.astype(np.int32)).cuda()
    ci[7] = n + 3
    va = torch.from_numpy(L.data).cuda()
    X = torch.zeros((n, k), dtype=torch.float64, device="cuda")
    ev = torch.zeros(k, dtype=torch.float64, device="cuda")
    g = torch.empty(L.nnz, dtype=torch.float64, device="cuda")
    rc = _native.lib.lg_eigsh_adjoint(n, L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr(), k, ev.data_ptr(),
                                      X.data_ptr(), None, None, g.data_ptr(), 10, 1e-10, None,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == _native.LG_ERR_INVALID
    assert "malformed CSR" in _native.last_error()


def test_plan_rejects_malformed_device_csr(torch_cuda):
    torch = torch_cuda
    import gpu_eigsh
    from oracle.adjoint import reference_test_laplacian

    L = reference_test_laplacian(50)
    n = L.shape[0]
    rp = torch.from_numpy(L.indptr.astype(np.int32)).cuda()
    ci = torch.from_numpy(L.indices.astype(np.int32)).cuda()
    ci[3] = -1
    va = torch.from_numpy(L.data).cuda()
    with pytest.raises(gpu_eigsh.LanczosError, match="column index out of range"):
        gpu_eigsh.EigshPlan(None, max_ncv=20, device_csr=(n, L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr()))
