"""CPU: pin the IRLM oracle against scipy ARPACK and analytic eigenvalues.

The reference's own forward test compares its IRLM with scipy
eigsh(which='SM', tol=1e-10) at rel. err < 1e-10 (tests/test_gradient.py:59-81)
on a kNN L_sym; the known-answer case is the Dirichlet grid Laplacian whose
eigenvalues are sum_d (2 - 2 cos(j_d pi/(N+1))).
"""
import numpy as np
import pytest
import scipy.sparse as sp

from gpu_eigsh import synthetic as syn
from oracle.irlm import arpack_eigsh, oracle_eigsh, oracle_lanczos_steps

from _parity import anorm1, eig_rel_err


def test_grid_known_answer_cfg0():
    # configuration 0: 100x100 Dirichlet grid, k=10 SA, ncv=40, tol=1e-10, v0 ~ N(0,1) seed 0
    L = syn.grid2d_dirichlet(100)
    assert L.shape == (10000, 10000) and L.nnz == 49600
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    (w, V), info = oracle_eigsh(L, 10, ncv=40, which="SA", tol=1e-10, v0=v0)
    exact = syn.grid_eigenvalues(100, 2)[:10]
    assert info["converged"]
    assert np.max(np.abs(w - exact) / exact) < 1e-10
    ws, _ = arpack_eigsh(L, 10, which="SA", ncv=40, tol=1e-10, v0=v0)
    assert np.max(np.abs(w - ws) / np.abs(ws)) < 1e-10
    res = np.linalg.norm(L @ V - V * w, axis=0)
    assert res.max() < 1e-8 * 8.0


@pytest.mark.parametrize("which", ["LA", "SA", "LM", "SM"])
def test_knn_which_vs_arpack(which):
    L, _ = syn.knn_laplacian(3000, k=10, seed=3)
    v0 = np.random.default_rng(5).standard_normal(L.shape[0])
    (w, V), info = oracle_eigsh(L, 8, ncv=30, which=which, tol=1e-10, v0=v0)
    ws, _ = arpack_eigsh(L, 8, which=which, ncv=30, tol=1e-10, v0=v0)
    assert info["converged"]
    assert eig_rel_err(w, ws, anorm1(L)) < 1e-10


def test_be_without_multiplicity():
    rng = np.random.default_rng(11)
    d = np.sort(rng.uniform(-3, 5, 1500))
    A = sp.diags(d) + sp.diags([0.01 * np.ones(1499)], [1]) + sp.diags([0.01 * np.ones(1499)], [-1])
    A = A.tocsr()
    v0 = rng.standard_normal(1500)
    (w, _), info = oracle_eigsh(A, 6, ncv=40, which="BE", tol=1e-10, v0=v0)
    ws, _ = arpack_eigsh(A, 6, which="BE", ncv=40, tol=1e-10, v0=v0)
    assert np.max(np.abs(w - ws) / np.abs(ws)) < 1e-10


def test_reference_dgks_vs_cgs2_same_tridiagonal():
    # Conditional DGKS (reference) and unconditional CGS2 (the CUDA engine) give
    # the same Lanczos tridiagonal to rounding.
    L, _ = syn.knn_laplacian(2000, k=10, seed=4)
    v0 = np.random.default_rng(1).standard_normal(L.shape[0])
    a1, b1 = oracle_lanczos_steps(L, 40, v0, cgs2=False)
    a2, b2 = oracle_lanczos_steps(L, 40, v0, cgs2=True)
    assert np.max(np.abs(a1 - a2)) < 1e-10 * np.abs(a1).max()
    assert np.max(np.abs(b1 - b2)) < 1e-10 * np.abs(b1).max()


def test_breakdown_invariant_subspace():
    # Block-diagonal matrix with a tiny block: the starting vector lives in a
    # 3-dimensional invariant subspace, so Lanczos breaks down after 3 steps.
    B = sp.diags([1.0, 2.0, 3.0])
    C = sp.diags(np.linspace(10, 20, 200))
    A = sp.block_diag([B, C]).tocsr()
    v0 = np.zeros(203)
    v0[:3] = [1.0, 1.0, 1.0]
    (w, _), info = oracle_eigsh(A, 4, ncv=20, which="SA", tol=1e-10, v0=v0)
    assert info["breakdowns"] >= 1
    np.testing.assert_allclose(w, [1.0, 2.0, 3.0, 10.0], rtol=1e-10)


@pytest.mark.parametrize("N", [1, 2, 5, 16])
def test_grid3d_device_builder_equals_host_builder(N):
    """The GPU-side assembly of the configuration-2 matrix (run here with torch
    on the CPU) gives the host builder's CSR exactly."""
    n, rp, col, val = syn.grid3d_dirichlet_device(N, device="cpu")
    B = syn.grid3d_dirichlet(N)
    B.eliminate_zeros()
    assert n == N ** 3 and int(rp[-1]) == 7 * n - 6 * N * N
    np.testing.assert_array_equal(rp.numpy(), B.indptr)
    np.testing.assert_array_equal(col.numpy(), B.indices)
    np.testing.assert_array_equal(val.numpy(), B.data)
