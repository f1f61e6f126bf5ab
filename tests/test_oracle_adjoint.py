"""Pins of the eigsh-backward oracle (oracle/adjoint.py) on CPU.

The reference's own implementation of this path (CUDA + LAPACK) cannot run
here, so the restatement is checked against known answers:
  * eigenvalue losses: the dense torch.linalg.eigh backward
    (Hellmann-Feynman, exact);
  * the deflated CG: the projected system solved densely;
  * eigenvector losses with k = 1 (where deflating against X drops nothing the
    loss sees, so the reference's gradient is the exact one): central finite
    differences of the dense eigendecomposition under symmetric perturbations.
"""
import numpy as np
import pytest
import torch

from oracle import adjoint as OA


def _dense_pairs(L, k):
    w, V = np.linalg.eigh(L.toarray())
    return w[:k], V[:, :k]


def test_eigenvalue_gradient_matches_dense_eigh_backward():
    L = OA.reference_test_laplacian(100)
    k = 5
    w, X = _dense_pairs(L, k)
    Ld = torch.from_numpy(L.toarray()).requires_grad_(True)
    ev, _ = torch.linalg.eigh(Ld)
    ev[1:k].sum().backward()
    dense = Ld.grad.numpy()
    g_evals = np.array([0.0, 1, 1, 1, 1])
    grad, iters = OA.adjoint_eigsh(L, w, X, g_evals=g_evals)
    rows = np.repeat(np.arange(L.shape[0]), np.diff(L.indptr))
    # eigh's backward symmetrises: (G + G^T)/2; the reference's entry-wise
    # gradient x x^T is already symmetric
    np.testing.assert_allclose(grad, dense[rows, L.indices], rtol=0, atol=1e-12)
    assert iters == [0] * k   # zero right-hand sides: no CG iterations


def test_deflated_cg_solves_the_projected_system():
    L = OA.reference_test_laplacian(120, seed=3)
    k = 6
    w, X = _dense_pairs(L, k)
    rng = np.random.default_rng(0)
    P = np.eye(L.shape[0]) - X @ X.T
    for i in range(k):
        b = OA.deflate(rng.standard_normal(L.shape[0]), X)
        x, it = OA.cg_deflated(L, w[i], b, X, tol=1e-12, max_iters=2000)
        assert it > 0
        M = P @ (L.toarray() - w[i] * np.eye(L.shape[0])) @ P
        ref = np.linalg.pinv(M, rcond=1e-10) @ b
        assert np.linalg.norm(x - ref) <= 1e-8 * np.linalg.norm(ref)


@pytest.mark.parametrize("idx", [0, 1])
def test_single_eigenvector_gradient_matches_finite_differences(idx):
    """k = 1: loss = (u . x)^2 for a fixed u (sign invariant)."""
    L = OA.reference_test_laplacian(60, nn=6, seed=5)
    n = L.shape[0]
    u = np.random.default_rng(1).standard_normal(n)
    w, V = np.linalg.eigh(L.toarray())
    x = V[:, idx]
    g_vec = (2.0 * (u @ x) * u)[:, None]
    grad, _ = OA.adjoint_eigsh(L, w[idx:idx + 1], x[:, None], g_evecs=g_vec, cg_tol=1e-13, cg_max_iters=5000)
    rows = np.repeat(np.arange(n), np.diff(L.indptr))
    pos = {(r, c): p for p, (r, c) in enumerate(zip(rows, L.indices))}
    rng = np.random.default_rng(2)
    h = 1e-6
    checked = 0
    for p in rng.choice(L.nnz, 40, replace=False):
        r, c = int(rows[p]), int(L.indices[p])
        E = np.zeros((n, n))
        E[r, c] += h
        if r != c:
            E[c, r] += h
        def loss(M):
            _, VV = np.linalg.eigh(M)
            return float((u @ VV[:, idx]) ** 2)
        fd = (loss(L.toarray() + E) - loss(L.toarray() - E)) / (2 * h)
        an = grad[p] + (grad[pos[(c, r)]] if r != c else 0.0)
        assert abs(fd - an) <= 1e-6 * max(1.0, abs(fd)), (r, c, fd, an)
        checked += 1
    assert checked == 40
