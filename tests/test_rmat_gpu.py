"""GPU: power-law matrices (configuration 4's family).

* rows longer than the row kernels' cut (kLongRow = 2048 nonzeros) are summed
  in chunks and combined in a fixed order: matvec and eigsh on a graph with hub
  rows of 3000 .. 9000 nonzeros match scipy / ARPACK;
* the R-MAT normalised Laplacian generated on the GPU
  (synthetic.rmat_laplacian_device) at scale 14, mixed precision (fp32 values,
  fp64 accumulation and basis), k=32 which='LA' ncv=96 tol=1e-8 as in
  configuration 4, matches ARPACK on the fp32-rounded matrix;
* the same with the rows renumbered by descending degree inside the plan
  (LG_PLAN_REORDER_DEGREE): eigenvalues, eigenvector residuals and the
  plan's matvec are those of the caller's matrix in the caller's numbering.
"""
import numpy as np
import pytest
import scipy.sparse as sp

from _parity import anorm1, eig_rel_err

pytestmark = pytest.mark.gpu


def _hub_laplacian(n=20000, hubs=(3000, 5000, 9000), seed=5):
    rng = np.random.default_rng(seed)
    src = rng.integers(0, n, 6 * n)
    dst = rng.integers(0, n, 6 * n)
    for h, deg in enumerate(hubs):
        nb = rng.choice(n, size=deg, replace=False)
        src = np.concatenate([src, np.full(deg, h)])
        dst = np.concatenate([dst, nb])
    lo, hi = np.minimum(src, dst), np.maximum(src, dst)
    keep = lo != hi
    key = np.unique(lo[keep] * n + hi[keep])
    from gpu_eigsh import synthetic as syn

    return syn.normalized_laplacian(n, key // n, key % n)


def test_long_rows_matvec_and_eigsh():
    import torch

    import gpu_eigsh
    from oracle.irlm import arpack_eigsh

    L = _hub_laplacian()
    lens = np.diff(L.indptr)
    assert (lens > 2048).sum() == 3 and lens.max() > 3 * 2048
    x = np.random.default_rng(1).standard_normal(L.shape[0])
    with gpu_eigsh.EigshPlan(L, max_ncv=40) as plan:
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        plan.matvec_device(xd.data_ptr(), yd.data_ptr())
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
    ref = L @ x
    assert np.abs(y - ref).max() <= 1e-13 * np.abs(ref).max()
    v0 = np.random.default_rng(2).standard_normal(L.shape[0])
    w, V = gpu_eigsh.gpu_eigsh(L, k=6, which="LA", ncv=30, tol=1e-10, v0=v0)
    ws, _ = arpack_eigsh(L, 6, which="LA", ncv=30, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, anorm1(L)) < 1e-10
    assert np.linalg.norm(L @ V - V * w, axis=0).max() <= 1e-10 * anorm1(L)


def test_rmat_scale14_mixed_config4_settings():
    import torch

    import gpu_eigsh
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    n, rp, col, val, info = syn.rmat_laplacian_device(14, device="cuda")
    L = sp.csr_matrix((val.cpu().numpy(), col.cpu().numpy(), rp.cpu().numpy()), shape=(n, n))
    assert abs(L - L.T).max() == 0.0
    L32 = L.astype(np.float32).astype(np.float64)
    v0 = np.random.default_rng(0).standard_normal(n)
    plan = gpu_eigsh.EigshPlan(None, max_ncv=96, mixed=True,
                               device_csr=(n, int(col.numel()), rp.data_ptr(), col.data_ptr(), val.data_ptr()))
    try:
        w, V = plan.solve(k=32, which="LA", ncv=96, tol=1e-8, v0=v0)
    finally:
        plan.close()
    ws, _ = arpack_eigsh(L32, 32, which="LA", ncv=96, tol=1e-8, v0=v0)
    assert eig_rel_err(w, ws, anorm1(L32)) < 1e-8
    assert np.linalg.norm(L32 @ V - V * w, axis=0).max() <= 1e-8 * anorm1(L32)
    torch.cuda.synchronize()


def test_rmat_degree_order_keeps_caller_numbering():
    import torch

    import gpu_eigsh
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    n, rp, col, val, info = syn.rmat_laplacian_device(14, device="cuda")
    L = sp.csr_matrix((val.cpu().numpy(), col.cpu().numpy(), rp.cpu().numpy()), shape=(n, n))
    L32 = L.astype(np.float32).astype(np.float64)
    v0 = np.random.default_rng(0).standard_normal(n)
    for mixed, M, tol in ((True, L32, 1e-8), (False, L, 1e-10)):
        plan = gpu_eigsh.EigshPlan(None, max_ncv=96, mixed=mixed, reorder="degree",
                                   device_csr=(n, int(col.numel()), rp.data_ptr(), col.data_ptr(), val.data_ptr()))
        try:
            w, V = plan.solve(k=32, which="LA", ncv=96, tol=tol, v0=v0)
            x = torch.from_numpy(v0).cuda()
            y = torch.empty_like(x)
            plan.matvec_device(x.data_ptr(), y.data_ptr())
            torch.cuda.synchronize()
            y = y.cpu().numpy()
        finally:
            plan.close()
        ref = M @ v0
        assert np.abs(y - ref).max() <= 1e-13 * np.abs(ref).max()
        ws, _ = arpack_eigsh(M, 32, which="LA", ncv=96, tol=tol, v0=v0)
        assert eig_rel_err(w, ws, anorm1(M)) < tol
        assert np.linalg.norm(M @ V - V * w, axis=0).max() <= tol * anorm1(M)


def test_degree_order_with_long_rows_matches_plain_plan():
    """Hub rows beyond the row kernels' cut keep their chunked sums under the
    degree numbering: same matvec to rounding, same eigenvalues."""
    import torch

    import gpu_eigsh

    L = _hub_laplacian()
    x = np.random.default_rng(1).standard_normal(L.shape[0])
    with gpu_eigsh.EigshPlan(L, max_ncv=40, reorder="degree") as plan:
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        plan.matvec_device(xd.data_ptr(), yd.data_ptr())
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        v0 = np.random.default_rng(2).standard_normal(L.shape[0])
        w, _ = plan.solve(k=6, which="LA", ncv=30, tol=1e-10, v0=v0)
    ref = L @ x
    assert np.abs(y - ref).max() <= 1e-13 * np.abs(ref).max()
    w0 = gpu_eigsh.gpu_eigsh(L, k=6, which="LA", ncv=30, tol=1e-10, v0=v0, return_eigenvectors=False)
    assert eig_rel_err(w, np.sort(w0), anorm1(L)) < 1e-10
