"""CPU oracle for the kNN graph builders — TEST INFRASTRUCTURE ONLY.

Restates, in numpy, the reference's two graph constructions so that the GPU
builder (lg_knn / lg_knn_laplacian_*) can be checked against them:

* ``knn_bruteforce`` — src/main.cu:42-63: for every point the squared
  distances to all others (coordinate order, one multiply and one add per
  coordinate), then the k smallest (dist2, j) pairs in pair order (the
  partial_sort over std::pair<double, int>).
* ``driver_laplacian`` — src/main.cu:59-107: weights exp(-d2 / (4 bw^2)),
  union symmetrisation (an edge listed by only one endpoint is added to the
  other with the same weight), rows sorted by column with the diagonal
  (degree = sequential sum of the row's weights in column order) at its
  sorted position, off-diagonals -w.
* ``generator_laplacian`` — benchmark/generate_large_laplacian.py:29-66:
  RandomState(seed).random((n, dim)), cKDTree.query(k + 1) with the first
  column dropped, the same weights from d**2, A.maximum(A.T), L = D - A.

Pins: ``generator_laplacian`` against the matrices the reference script
itself wrote (tests/golden/make_graph_golden.py ->
tests/golden/graph_generator.npz), and ``driver_laplacian`` against
``generator_laplacian`` on the same points (tests/test_oracle_graph.py).
"""
from __future__ import annotations

import numpy as np


def sq_dists(pts: np.ndarray, i: int) -> np.ndarray:
    """Squared distances from point i to all points, summed in coordinate order."""
    s = np.zeros(pts.shape[0])
    for d in range(pts.shape[1]):
        t = pts[:, d] - pts[i, d]
        s = s + t * t
    return s


def knn_bruteforce(pts: np.ndarray, k: int):
    """(idx (n, k) int64, d2 (n, k)) ascending by (d2, index), self excluded."""
    pts = np.ascontiguousarray(pts, dtype=np.float64)
    n = pts.shape[0]
    idx = np.empty((n, k), dtype=np.int64)
    d2 = np.empty((n, k))
    cand = np.arange(n)
    for i in range(n):
        s = sq_dists(pts, i)
        keep = cand != i
        order = np.lexsort((cand[keep], s[keep]))[:k]
        idx[i] = cand[keep][order]
        d2[i] = s[keep][order]
    return idx, d2


def driver_laplacian(idx: np.ndarray, d2: np.ndarray, bw: float):
    """L = D - A from neighbour lists, src/main.cu:59-107.  Returns
    (indptr, indices, data) of the CSR."""
    n, k = idx.shape
    nbrs = [dict() for _ in range(n)]
    for i in range(n):
        for q in range(k):
            nbrs[i][int(idx[i, q])] = float(np.exp(-d2[i, q] / (4.0 * bw * bw)))
    for i in range(n):
        for j, w in list(nbrs[i].items())[:k]:
            if i not in nbrs[j]:
                nbrs[j][i] = w
    indptr = np.zeros(n + 1, dtype=np.int64)
    cols, vals = [], []
    for i in range(n):
        row = sorted(nbrs[i].items())
        deg = 0.0
        for _, w in row:
            deg += w
        entries = [(j, -w) for j, w in row] + [(i, deg)]
        entries.sort(key=lambda t: t[0])
        cols.extend(j for j, _ in entries)
        vals.extend(v for _, v in entries)
        indptr[i + 1] = len(cols)
    return indptr, np.array(cols, dtype=np.int64), np.array(vals)


def generator_points(n: int, dim: int, seed: int) -> np.ndarray:
    return np.random.RandomState(seed).random((n, dim))


def generator_laplacian(n: int, dim: int, k: int, bw: float, seed: int):
    """scipy CSR of the reference generator's matrix."""
    import scipy.sparse as sp
    from scipy.spatial import cKDTree

    pts = generator_points(n, dim, seed)
    dist, ind = cKDTree(pts).query(pts, k=k + 1)
    dist, ind = dist[:, 1:], ind[:, 1:]
    w = np.exp(-dist ** 2 / (4.0 * bw ** 2))
    A = sp.csr_matrix((w.ravel(), (np.repeat(np.arange(n), k), ind.ravel())), shape=(n, n))
    A = A.maximum(A.T)
    deg = np.array(A.sum(axis=1)).ravel()
    L = sp.csr_matrix((deg, (np.arange(n), np.arange(n))), shape=(n, n)) - A
    L = L.tocsr()
    L.sort_indices()
    return L
