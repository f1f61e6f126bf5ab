"""GPU parity tests of the eigsh path (CUDA engine through the C ABI).

Tolerances: eigenvalues match scipy ARPACK to 1e-10 relative (fp64), every
Ritz pair satisfies ||A v - lambda v|| <= tol * ||A|| (the north-star targets),
and the Lanczos tridiagonal matches the CPU oracle step by step.
"""
import ctypes

import numpy as np
import pytest
import scipy.sparse as sp

from _parity import anorm1, eig_rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ge():
    import gpu_eigsh

    return gpu_eigsh


def _residuals(A, w, V):
    return np.linalg.norm(A @ V - V * w, axis=0)


def test_cfg0_grid_known_answer(ge):
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    L = syn.grid2d_dirichlet(100)
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    w, V = ge.gpu_eigsh(L, k=10, which="SA", ncv=40, tol=1e-10, v0=v0)
    exact = syn.grid_eigenvalues(100, 2)[:10]
    assert eig_rel_err(w, exact, 8.0) < 1e-10
    ws, _ = arpack_eigsh(L, 10, which="SA", ncv=40, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, 8.0) < 1e-10
    assert _residuals(L, w, V).max() <= 1e-10 * 8.0
    np.testing.assert_allclose(V.T @ V, np.eye(10), atol=1e-10)


@pytest.mark.parametrize("which", ["LA", "SA", "LM", "SM"])
def test_knn_which_vs_arpack(ge, which):
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    L, _ = syn.knn_laplacian(5000, k=10, seed=3)
    an = anorm1(L)
    v0 = np.random.default_rng(5).standard_normal(L.shape[0])
    w, V = ge.gpu_eigsh(L, k=8, which=which, ncv=30, tol=1e-10, v0=v0)
    ws, Vs = arpack_eigsh(L, 8, which=which, ncv=30, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, an) < 1e-10
    assert _residuals(L, w, V).max() <= 1e-10 * an
    # same invariant subspace (spectrum here has no multiplicities)
    s = np.linalg.svd(V.T @ Vs, compute_uv=False)
    assert s.min() > 1 - 1e-8


def test_be_without_multiplicity(ge):
    from oracle.irlm import arpack_eigsh

    rng = np.random.default_rng(11)
    d = np.sort(rng.uniform(-3, 5, 1500))
    A = (sp.diags(d) + sp.diags([0.01 * np.ones(1499)], [1]) + sp.diags([0.01 * np.ones(1499)], [-1])).tocsr()
    v0 = rng.standard_normal(1500)
    w, _ = ge.gpu_eigsh(A, k=6, which="BE", ncv=40, tol=1e-10, v0=v0)
    ws, _ = arpack_eigsh(A, 6, which="BE", ncv=40, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, anorm1(A)) < 1e-10


def test_factorization_matches_oracle_step_by_step(ge):
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import oracle_lanczos_steps

    L, _ = syn.knn_laplacian(20000, k=10, seed=7)
    v0 = np.random.default_rng(2).standard_normal(L.shape[0])
    with ge.EigshPlan(L, max_ncv=64) as plan:
        a, b = plan.factorize(v0, 60)
    ao, bo = oracle_lanczos_steps(L, 60, v0, cgs2=True)
    scale = np.abs(ao).max()
    assert np.max(np.abs(a - ao)) < 1e-12 * scale
    assert np.max(np.abs(b[1:] - bo[1:])) < 1e-12 * scale


def test_mixed_precision_vs_fp32_rounded_matrix(ge):
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    L, _ = syn.knn_laplacian(8000, k=10, seed=9)
    L32 = L.astype(np.float32).astype(np.float64)
    v0 = np.random.default_rng(3).standard_normal(L.shape[0])
    w, V = ge.gpu_eigsh(L, k=10, which="LA", ncv=30, tol=1e-10, v0=v0, mixed=True)
    ws, _ = arpack_eigsh(L32, 10, which="LA", ncv=30, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, anorm1(L32)) < 1e-10


def _reference_test_laplacian(n, nn=10, seed=42):
    # L_sym of a kNN graph on N(0, I_5) points — the matrix family of the
    # reference's forward test (tests/test_gradient.py:26-45), rebuilt here.
    from scipy.spatial import cKDTree

    rng = np.random.RandomState(seed)
    pts = rng.randn(n, 5)
    d, idx = cKDTree(pts).query(pts, k=nn + 1)
    rows = np.repeat(np.arange(n), nn)
    A = sp.csr_matrix((np.exp(-d[:, 1:] ** 2 / 4.0).ravel(), (rows, idx[:, 1:].ravel())), shape=(n, n))
    A = A.maximum(A.T)
    deg = np.asarray(A.sum(axis=1)).ravel()
    Dm = sp.diags(1.0 / np.sqrt(np.maximum(deg, 1e-15)))
    return (Dm @ (sp.diags(deg) - A) @ Dm).tocsr()


def test_reference_abi_compute_eigsh(ge):
    from gpu_eigsh import _native
    from scipy.sparse.linalg import eigsh

    L = _reference_test_laplacian(500)
    k = 10
    ip = np.ascontiguousarray(L.indptr, dtype=np.int32)
    ix = np.ascontiguousarray(L.indices, dtype=np.int32)
    dv = np.ascontiguousarray(L.data, dtype=np.float64)
    evals = np.zeros(k)
    evecs = np.zeros(500 * k)
    PI, PD = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)
    rc = _native.lib.compute_eigsh(500, L.nnz, ip.ctypes.data_as(PI), ix.ctypes.data_as(PI), dv.ctypes.data_as(PD),
                                   k, 0, 2000, 1e-12, evals.ctypes.data_as(PD), evecs.ctypes.data_as(PD))
    assert rc == k
    ws = np.sort(eigsh(L, k=k, which="SM", tol=1e-10)[0])
    assert np.max(np.abs(evals[1:] - ws[1:]) / np.abs(ws[1:])) < 1e-10
    V = evecs.reshape(k, 500).T   # column-major n x k
    assert _residuals(L, evals, V).max() < 1e-9


def test_shift_invert_vs_arpack(ge):
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    L = syn.grid2d_dirichlet(60)
    v0 = np.random.default_rng(4).standard_normal(L.shape[0])
    w, V = ge.gpu_eigsh(L, k=6, sigma=0.0, ncv=24, tol=1e-10, v0=v0, cg_tol=1e-13, cg_max_iters=5000)
    ws, _ = arpack_eigsh(L, 6, sigma=0.0, ncv=24, tol=1e-10, v0=v0)
    assert eig_rel_err(w, ws, 8.0) < 1e-9
    assert _residuals(L, w, V).max() < 1e-8


def test_reference_abi_shift_invert(ge):
    from gpu_eigsh import _native
    from scipy.sparse.linalg import eigsh

    L = _reference_test_laplacian(500) + 1e-3 * sp.identity(500)
    L = L.tocsr()
    k = 6
    ip = np.ascontiguousarray(L.indptr, dtype=np.int32)
    ix = np.ascontiguousarray(L.indices, dtype=np.int32)
    dv = np.ascontiguousarray(L.data, dtype=np.float64)
    evals = np.zeros(k)
    PI, PD = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)
    rc = _native.lib.compute_eigsh_sigma(500, L.nnz, ip.ctypes.data_as(PI), ix.ctypes.data_as(PI),
                                         dv.ctypes.data_as(PD), k, 0, 4000, 1e-10, 0.0, 5000, 1e-12,
                                         evals.ctypes.data_as(PD), None)
    assert rc == k
    ws = np.sort(eigsh(L, k=k, sigma=0.0, tol=1e-10)[0])
    assert np.max(np.abs(evals - ws) / np.abs(ws)) < 1e-8


def test_invariant_subspace_breakdown(ge):
    B = sp.diags([1.0, 2.0, 3.0])
    C = sp.diags(np.linspace(10, 20, 200))
    A = sp.block_diag([B, C]).tocsr()
    v0 = np.zeros(203)
    v0[:3] = 1.0
    (w, V), info = ge.gpu_eigsh(A, k=4, which="SA", ncv=20, tol=1e-10, v0=v0, return_info=True)
    assert info["breakdowns"] >= 1
    np.testing.assert_allclose(w, [1.0, 2.0, 3.0, 10.0], rtol=1e-10)
    assert _residuals(A, w, V).max() < 1e-9


def test_no_convergence_raises_scipy_exception(ge):
    from gpu_eigsh import synthetic as syn

    L, _ = syn.knn_laplacian(4000, k=10, seed=1)
    with pytest.raises(ge.ArpackNoConvergence) as ei:
        ge.gpu_eigsh(L, k=10, which="SA", ncv=22, tol=1e-14, maxiter=1)
    assert ei.value.eigenvalues.shape == (10,)


def test_argument_errors(ge):
    from gpu_eigsh import synthetic as syn

    L = syn.grid2d_dirichlet(10)
    with pytest.raises(ValueError):
        ge.gpu_eigsh(L, k=0)
    with pytest.raises(TypeError):
        ge.gpu_eigsh(L, k=100)
    with pytest.raises(ValueError):
        ge.gpu_eigsh(L, k=5, ncv=5)
    with pytest.raises(ValueError):
        ge.gpu_eigsh(L, k=5, which="XX")
    with pytest.raises(ValueError):
        ge.gpu_eigsh(L, k=5, v0=np.zeros(100))
    bad = L.copy()
    bad.data[3] = np.nan
    with pytest.raises(ge.LanczosError):
        ge.gpu_eigsh(bad, k=5)


def test_bitwise_repeatable(ge):
    from gpu_eigsh import synthetic as syn

    L, _ = syn.knn_laplacian(30000, k=10, seed=5)
    a = ge.gpu_eigsh(L, k=10, which="LA", ncv=30, tol=1e-10)
    b = ge.gpu_eigsh(L, k=10, which="LA", ncv=30, tol=1e-10)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_profile_mode_accounts_every_launch(ge):
    """Profile mode (CUDA events around every launch; what the bench's
    rooflines read) changes no result, and its record is consistent: every
    launch of the solve is in some kernel class, the single-GPU plan spends
    nothing in the multi-GPU class, and the bytes of the sparse product are
    its per-launch formula times its launches."""
    from gpu_eigsh import synthetic as syn

    L, _ = syn.knn_laplacian(40000, k=10, seed=8)
    n, nnz = L.shape[0], L.nnz
    v0 = np.random.default_rng(2).standard_normal(n)
    plan = ge.EigshPlan(L, max_ncv=40)
    try:
        w0, V0 = plan.solve(k=10, which="LA", ncv=30, tol=1e-10, v0=v0)
        plain = dict(plan.last_info)
        w1, V1 = plan.solve(k=10, which="LA", ncv=30, tol=1e-10, v0=v0, profile=True)
        prof = dict(plan.last_info)
    finally:
        plan.close()
    assert np.array_equal(w0, w1) and np.array_equal(V0, V1)
    assert prof["steps"] == plain["steps"] and prof["launches"] == plain["launches"]
    calls, ms, by = prof["kernel_calls"], prof["kernel_ms"], prof["kernel_bytes"]
    assert sum(calls.values()) <= prof["launches"]
    for cls in ("spmv", "gs_project", "gs_correct_project", "restart", "basis"):
        assert calls[cls] > 0 and ms[cls] > 0.0, cls
    assert calls["comm"] == 0 and ms["comm"] == 0.0
    # lag steps: (4 + 8) nnz + 4 (n + 1) + 8n (x) + 8n (z) per launch; the
    # first step of each extension (in-step passes) writes v_j too (+8n)
    lo = calls["spmv"] * ((12.0 * nnz + 4.0 * (n + 1) + 16.0 * n))
    hi = calls["spmv"] * ((12.0 * nnz + 4.0 * (n + 1) + 24.0 * n))
    assert lo <= by["spmv"] <= hi
    assert sum(ms.values()) < 5.0 * prof["ms"]


def test_device_pointer_api_with_torch(ge):
    import torch
    from gpu_eigsh import synthetic as syn

    L, _ = syn.knn_laplacian(20000, k=10, seed=6)
    dev = torch.device("cuda")
    rp = torch.from_numpy(L.indptr.astype(np.int32)).to(dev)
    ci = torch.from_numpy(L.indices.astype(np.int32)).to(dev)
    va = torch.from_numpy(L.data).to(dev)
    v0 = torch.from_numpy(np.random.default_rng(1).standard_normal(L.shape[0])).to(dev)
    Y = torch.empty((L.shape[0], 6), dtype=torch.float64, device=dev)
    torch.cuda.synchronize()
    plan = ge.EigshPlan(None, max_ncv=40, device_csr=(L.shape[0], L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr()))
    w, _ = plan.solve(k=6, which="LA", ncv=30, tol=1e-10, v0_device=v0.data_ptr(), evecs_out=Y.data_ptr())
    plan.close()
    w2, V2 = ge.gpu_eigsh(L, k=6, which="LA", ncv=30, tol=1e-10, v0=v0.cpu().numpy())
    np.testing.assert_allclose(w, w2, rtol=1e-12)
    np.testing.assert_allclose(np.abs(Y.cpu().numpy()), np.abs(V2), atol=1e-8)


def test_knn_1e6_properties(ge):
    """Configuration 1 at full size: n = 1e6 kNN Laplacian, k=20 LA, ncv=60,
    tol=1e-10.  Checked through size-independent properties (every residual
    <= tol*||A||, orthonormal eigenvectors) and against the mixed mode."""
    from gpu_eigsh import synthetic as syn

    L, info = syn.knn_laplacian(1_000_000, k=10, seed=1)
    an = anorm1(L)
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    (w, V), inf = ge.gpu_eigsh(L, k=20, which="LA", ncv=60, tol=1e-10, v0=v0, return_info=True)
    res = _residuals(L, w, V)
    assert res.max() <= 1e-10 * an
    G = V.T @ V
    assert np.abs(G - np.eye(20)).max() < 1e-9
    assert np.all(np.diff(w) >= 0)


def test_cfg2_shift_invert_grid3d_full_size(ge):
    """Configuration 2 at full size: 7-point Dirichlet Laplacian on 128^3
    (n = 2,097,152), sigma = 0, k = 16, ncv = 48, tol = 1e-10, inner CG to
    1e-12.  The spectrum is known in closed form: every eigenvalue must be an
    analytic one to 1e-10 relative, no distinct analytic eigenvalue below the
    largest one returned may be missing (single-vector Lanczos sees one
    direction per multiple eigenvalue until rounding seeds the others, so
    multiplicities may be incomplete, never the distinct values), and every
    pair satisfies ||A y - lambda y|| <= 1e-8 ||A||."""
    import torch

    from gpu_eigsh import synthetic as syn

    N = 128
    n, rp, col, val = syn.grid3d_dirichlet_device(N, device="cuda")
    assert int(col.numel()) == 14_581_760
    plan = ge.EigshPlan(None, max_ncv=48, device_csr=(n, int(col.numel()), rp.data_ptr(), col.data_ptr(),
                                                       val.data_ptr()))
    v0 = torch.from_numpy(np.random.default_rng(0).standard_normal(n)).cuda()
    Y = torch.empty((n, 16), dtype=torch.float64, device="cuda")
    w, _ = plan.solve(k=16, sigma=0.0, ncv=48, tol=1e-10, cg_tol=1e-12, v0_device=v0.data_ptr(),
                      evecs_out=Y.data_ptr())
    info = dict(plan.last_info)
    exact = syn.grid_eigenvalues(N, 3)[:200]
    near = exact[np.abs(exact[None, :] - w[:, None]).argmin(1)]
    assert np.max(np.abs(w - near) / near) < 1e-10, (w, near)
    distinct = np.unique(np.round(exact / exact[0], 9)) * exact[0]
    below = distinct[distinct <= w.max() * (1 + 1e-9)]
    for lam in below:
        assert np.min(np.abs(w - lam)) <= 1e-9 * lam, (lam, w)
    AY = torch.empty(n, dtype=torch.float64, device="cuda")
    for i in range(16):
        y = Y[:, i].contiguous()
        plan.matvec_device(y.data_ptr(), AY.data_ptr())
        assert float(torch.linalg.norm(AY - w[i] * y)) <= 1e-8 * 12.0
    G = Y.T @ Y
    assert float((G - torch.eye(16, dtype=torch.float64, device="cuda")).abs().max()) < 1e-9
    assert info["cg_failures"] == 0 and info["cg_iters"] > 0
    plan.close()


def test_plan_reorder_bfs_keeps_caller_numbering(ge):
    """LG_PLAN_REORDER_BFS: the plan renumbers the rows by BFS level inside;
    eigenvalues match ARPACK at 1e-10, the eigenvectors come back in the
    caller's numbering (residuals against the caller's matrix), matvec maps
    both ways, and the Lanczos tridiagonal equals the unordered plan's."""
    import torch

    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    L, _ = syn.knn_laplacian(20000, k=10, seed=7)
    v0 = np.random.default_rng(2).standard_normal(L.shape[0])
    an = anorm1(L)
    for mixed in (False, True):
        with ge.EigshPlan(L, max_ncv=40, mixed=mixed, reorder=True) as plan:
            w, V = plan.solve(k=8, which="LA", ncv=40, tol=1e-10, v0=v0)
            if not mixed:
                ws, _ = arpack_eigsh(L, 8, which="LA", ncv=40, tol=1e-10, v0=v0)
                assert eig_rel_err(w, ws, an) < 1e-10
                assert _residuals(L, w, V).max() <= 1e-10 * an
            x = torch.from_numpy(v0).cuda()
            y = torch.empty_like(x)
            plan.matvec_device(x.data_ptr(), y.data_ptr())
            Lx = (L.astype(np.float32).astype(np.float64) if mixed else L) @ v0
            assert np.abs(y.cpu().numpy() - Lx).max() <= 1e-12 * np.abs(Lx).max()
            a1, b1 = plan.factorize(v0, 20)
        with ge.EigshPlan(L, max_ncv=40, mixed=mixed) as plain:
            a0, b0 = plain.factorize(v0, 20)
        assert np.abs(a1 - a0).max() < 1e-10 * an and np.abs(b1 - b0).max() < 1e-10 * an


@pytest.mark.parametrize("case", ["knn_LA", "knn_SA", "grid_SA", "mixed_LA", "breakdown"])
def test_lag_steps_match_inline_cgs2(ge, case):
    """Delayed second Gram-Schmidt pass (the default) against both passes
    inside every step (LG_PLAN_CGS2_INLINE): the same eigenvalues to 1e-11
    relative, both at ARPACK's to 1e-10, residuals within tol * ||A||, an
    orthonormal Ritz basis, and the same restart count (to one restart)."""
    from gpu_eigsh import synthetic as syn
    from oracle.irlm import arpack_eigsh

    mixed = case == "mixed_LA"
    if case.startswith("knn") or mixed:
        A, _ = syn.knn_laplacian(20000, k=10, seed=11)
        k, which, ncv = 8, case.split("_")[1], 40
    elif case == "grid_SA":
        A, k, which, ncv = syn.grid2d_dirichlet(60), 10, "SA", 40
    else:
        A = sp.block_diag([sp.diags([1.0, 2.0, 3.0]), sp.diags(np.linspace(10, 20, 200))]).tocsr()
        k, which, ncv = 4, "SA", 20
    n = A.shape[0]
    v0 = np.random.default_rng(3).standard_normal(n)
    if case == "breakdown":
        v0[3:] = 0.0
    an = anorm1(A)
    out = {}
    for inline in (False, True):
        with ge.EigshPlan(A, max_ncv=ncv, mixed=mixed, cgs2_inline=inline) as plan:
            w, V = plan.solve(k=k, which=which, ncv=ncv, tol=1e-10, v0=v0)
            out[inline] = (w, V, dict(plan.last_info))
    (w0, V0, i0), (w1, V1, i1) = out[False], out[True]
    assert eig_rel_err(w0, w1, an) < 1e-11
    # the same Krylov spaces to rounding; a borderline convergence test may flip by one restart
    assert abs(i0["restarts"] - i1["restarts"]) <= 1
    Aref = A.astype(np.float32).astype(np.float64) if mixed else A
    assert _residuals(Aref, w0, V0).max() <= 1e-10 * an
    np.testing.assert_allclose(V0.T @ V0, np.eye(k), atol=1e-10)
    if not mixed:
        ws, _ = arpack_eigsh(A, k, which=which, ncv=ncv, tol=1e-10, v0=v0)
        assert eig_rel_err(w0, ws, an) < 1e-10
    if case == "breakdown":
        assert i0["breakdowns"] >= 1
        np.testing.assert_allclose(w0, [1.0, 2.0, 3.0, 10.0], rtol=1e-10)
    else:
        assert i0["launches"] < i1["launches"]   # one stream of the basis fewer per step
