"""CPU (numpy) restatement of the reference's eigsh backward (implicit
differentiation of the eigenpairs).

TEST INFRASTRUCTURE ONLY: imported by tests/ to check results; the product path
never imports it.  The reference's own code for this path is CUDA + LAPACK and
cannot run here, so the restatement is pinned by known answers instead
(tests/test_oracle_adjoint.py): eigenvalue losses against the dense
torch.linalg.eigh backward (Hellmann-Feynman: d lambda_i / dA = x_i x_i^T) and
eigenvector losses against central finite differences of the dense
eigendecomposition, both on the reference's test matrix construction
(tests/test_gradient.py:27-48 of the reference).

Follows (reference file:line):
  deflate_against (v -= X X^T v) ........... src/inner_solve.cuh:69-84
  deflated CG on (A - sigma I) x = b ....... src/inner_solve.cuh:110-200
  compute_adjoint_eigsh: per pair i,
    rhs = (I - X X^T) g_vec_i, CG solve,
    xi re-deflated, grad_vals[p] +=
    (g_val_i x_i[r] - xi[r]) x_i[c] ........ python/gpu_eigsh/_cuda_eigsh.cu:183-326
  differentiable_eigsh defaults ........... python/gpu_eigsh/differentiable.py:120-202
"""
from __future__ import annotations

import numpy as np

SAFE_MIN = np.finfo(np.float64).tiny


def deflate(v, X):
    return v - X @ (X.T @ v)


def cg_deflated(A, sigma, b, X, tol=1e-10, max_iters=500):
    """(A - sigma I) x = b with x, r kept orthogonal to span(X); returns
    (x, iterations; negative when the iteration limit or a breakdown ended it)."""
    x = np.zeros_like(b)
    r = deflate(b.copy(), X)
    p = r.copy()
    rr_old = float(r @ r)
    bnorm = float(np.linalg.norm(b))
    if bnorm < SAFE_MIN:
        return x, 0
    tol_abs = tol * bnorm
    for it in range(max_iters):
        Ap = A @ p - sigma * p
        Ap = deflate(Ap, X)
        pAp = float(p @ Ap)
        if abs(pAp) < SAFE_MIN:
            return x, -(it + 1)
        alpha = rr_old / pAp
        x = x + alpha * p
        r = r - alpha * Ap
        r = deflate(r, X)
        rr_new = float(r @ r)
        if np.sqrt(rr_new) < tol_abs:
            return deflate(x, X), it + 1
        beta = rr_new / rr_old
        p = r + beta * p
        rr_old = rr_new
    return deflate(x, X), -max_iters


def adjoint_eigsh(A, evals, X, g_evals=None, g_evecs=None, cg_max_iters=500, cg_tol=1e-10):
    """Gradient with respect to the stored values of the CSR matrix A
    (scipy.sparse, sorted or not: one output per stored entry, in storage
    order).  X: n x k eigenvectors (columns).  Returns (grad_vals, iterations
    per pair)."""
    A = A.tocsr()
    n, k = X.shape
    rows = np.repeat(np.arange(n), np.diff(A.indptr))
    cols = A.indices
    grad = np.zeros(A.nnz)
    iters = []
    for i in range(k):
        gv = np.zeros(n) if g_evecs is None else np.asarray(g_evecs[:, i], dtype=np.float64)
        rhs = deflate(gv.copy(), X)
        xi, it = cg_deflated(A, float(evals[i]), rhs, X, cg_tol, cg_max_iters)
        iters.append(it)
        xi = deflate(xi, X)
        ge = 0.0 if g_evals is None else float(g_evals[i])
        coeff = ge * X[:, i] - xi
        grad += coeff[rows] * X[cols, i]
    return grad, iters


def reference_test_laplacian(n, nn=10, seed=42):
    """The symmetric-normalised kNN Laplacian the reference's gradient tests
    build (tests/test_gradient.py:27-48): 5-D Gaussian points (numpy global
    seed), nn neighbours, weights exp(-d^2/4), union-symmetrised."""
    import scipy.sparse as sp
    from scipy.spatial import cKDTree

    rng = np.random.RandomState(seed)
    points = rng.randn(n, 5)
    d, ix = cKDTree(points).query(points, k=nn + 1)
    rows = np.repeat(np.arange(n), nn)
    W = sp.csr_matrix((np.exp(-d[:, 1:] ** 2 / 4.0).ravel(), (rows, ix[:, 1:].ravel())), shape=(n, n))
    W = W.maximum(W.T)
    deg = np.asarray(W.sum(axis=1)).ravel()
    Dm = sp.diags(1.0 / np.sqrt(np.maximum(deg, 1e-15)))
    L = Dm @ (sp.diags(deg) - W) @ Dm
    L = L.tocsr()
    L.sort_indices()
    return L
