"""Seeded synthetic workloads for the Lanczos hot path.

The reference measures only on seeded synthetic graphs (no public dataset);
these builders produce the same families at the sizes used for parity tests
and benchmarks.  All are deterministic functions of their arguments.

* ``grid2d_dirichlet(N)``  — 5-point Dirichlet Laplacian on an N x N grid,
  kron(I, T) + kron(T, I), T = tridiag(-1, 2, -1); analytic eigenvalues
  ``grid_eigenvalues``.
* ``grid3d_dirichlet(N)``  — 7-point Dirichlet Laplacian on N^3
  (``grid3d_dirichlet_device``: the same matrix assembled on the GPU).
* ``knn_laplacian(n, k, seed)`` — points uniform in [0,1]^2, k nearest
  neighbours (self dropped), symmetrised by union (max(A, A^T), as the
  reference's benchmark/generate_large_laplacian.py:60 does), weights
  exp(-d^2 / 2h^2) with h the median k-th neighbour distance, L = D - W.
* ``knn_edge_list(n, k, seed)`` — the undirected edges (i < j) of that graph
  with squared lengths, in the IMGP operator's edge-list format
  (python/gpu_eigsh/imgp.py: idx (2, M) int64, x_edge_dists (M,)).
* ``rmat_edges(scale, edge_factor, abcd, seed)`` — R-MAT generator
  (Chakrabarti, Zhan, Faloutsos 2004), symmetrised, duplicates and
  self-loops removed; ``normalized_laplacian`` builds I - D^-1/2 W D^-1/2.
"""
from __future__ import annotations

import numpy as np
import scipy.sparse as sp


def _tridiag_t(N: int) -> sp.csr_matrix:
    e = np.ones(N)
    return sp.diags([-e[:-1], 2.0 * e, -e[:-1]], [-1, 0, 1], format="csr")


def grid2d_dirichlet(N: int) -> sp.csr_matrix:
    T = _tridiag_t(N)
    I = sp.identity(N, format="csr")
    L = (sp.kron(I, T) + sp.kron(T, I)).tocsr()
    L.sum_duplicates()
    L.sort_indices()
    return L


def grid3d_dirichlet(N: int) -> sp.csr_matrix:
    T = _tridiag_t(N)
    I = sp.identity(N, format="csr")
    L = (sp.kron(sp.kron(I, I), T) + sp.kron(sp.kron(I, T), I) + sp.kron(sp.kron(T, I), I)).tocsr()
    L.sum_duplicates()
    L.sort_indices()
    return L


def grid3d_dirichlet_device(N: int, device=None):
    """grid3d_dirichlet(N) assembled on the GPU with torch (configuration 2:
    N = 128, n = 2,097,152, nnz = 7n - 6N^2).  Vertex (z, y, x) is row
    z*N^2 + y*N + x; its row holds -1 at the in-grid neighbours and 6 on the
    diagonal, columns ascending.  Returns (n, rowptr int32, col int32,
    val float64) device tensors."""
    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    n = N ** 3
    i = torch.arange(n, device=dev, dtype=torch.int64)
    x, y, z = i % N, (i // N) % N, i // (N * N)
    # offsets in ascending column order, with the test that keeps each in the grid
    offs = [(-N * N, z > 0), (-N, y > 0), (-1, x > 0), (0, None), (1, x < N - 1), (N, y < N - 1),
            (N * N, z < N - 1)]
    cols, vals, keep = [], [], []
    for off, ok in offs:
        cols.append(i + off)
        vals.append(torch.full((n,), 6.0 if off == 0 else -1.0, dtype=torch.float64, device=dev))
        keep.append(torch.ones(n, dtype=torch.bool, device=dev) if ok is None else ok)
    C = torch.stack(cols, 1)
    Vv = torch.stack(vals, 1)
    K = torch.stack(keep, 1)
    counts = K.sum(1)
    rowptr = torch.zeros(n + 1, dtype=torch.int32, device=dev)
    rowptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    col = C[K].to(torch.int32)
    val = Vv[K]
    return n, rowptr, col, val


def grid_eigenvalues(N: int, dim: int) -> np.ndarray:
    """All eigenvalues of the dim-D Dirichlet grid Laplacian, ascending:
    sum_d (2 - 2 cos(j_d pi / (N+1))), j_d = 1..N."""
    lam1 = 2.0 - 2.0 * np.cos(np.arange(1, N + 1) * np.pi / (N + 1))
    out = lam1
    for _ in range(dim - 1):
        out = (out[:, None] + lam1[None, :]).ravel()
    return np.sort(out)


def _knn(n: int, k: int, seed: int, dim: int = 2):
    from scipy.spatial import cKDTree

    pts = np.random.default_rng(seed).uniform(size=(n, dim))
    tree = cKDTree(pts)
    d, idx = tree.query(pts, k=k + 1, workers=-1)
    return pts, d[:, 1:], idx[:, 1:]


def knn_laplacian(n: int, k: int = 10, seed: int = 1, dim: int = 2):
    """Returns (L csr float64, info dict)."""
    _, d, idx = _knn(n, k, seed, dim)
    h = float(np.median(d[:, k - 1]))
    w = np.exp(-(d ** 2) / (2.0 * h * h))
    rows = np.repeat(np.arange(n, dtype=np.int64), k)
    A = sp.csr_matrix((w.ravel(), (rows, idx.ravel())), shape=(n, n))
    A = A.maximum(A.T).tocsr()
    deg = np.asarray(A.sum(axis=1)).ravel()
    L = (sp.diags(deg) - A).tocsr()
    L.sum_duplicates()
    L.sort_indices()
    info = {"n": n, "k": k, "seed": seed, "h": h, "nnz": int(L.nnz), "edges": int((A.nnz) // 2)}
    return L, info


def knn_edge_list(n: int, k: int = 10, seed: int = 1, dim: int = 2):
    """Undirected edges (i < j) of the union-symmetrised kNN graph.
    Returns (idx (2, M) int64, d2 (M,) float64)."""
    _, d, idx = _knn(n, k, seed, dim)
    rows = np.repeat(np.arange(n, dtype=np.int64), k)
    cols = idx.ravel().astype(np.int64)
    d2 = (d ** 2).ravel()
    lo = np.minimum(rows, cols)
    hi = np.maximum(rows, cols)
    key = lo * n + hi
    order = np.argsort(key, kind="stable")
    key, d2 = key[order], d2[order]
    first = np.ones(key.shape[0], dtype=bool)
    first[1:] = key[1:] != key[:-1]
    key, d2 = key[first], d2[first]
    idx2 = np.stack([key // n, key % n]).astype(np.int64)
    return idx2, d2


def rmat_edges(scale: int, edge_factor: int = 16, abcd=(0.57, 0.19, 0.19, 0.05), seed: int = 2,
               chunk: int = 1 << 24):
    """R-MAT edges, symmetrised, without duplicates and self-loops.
    Returns (src, dst) int64 arrays with src < dst."""
    a, b, c, _ = abcd
    n = 1 << scale
    m = edge_factor * n
    rng = np.random.default_rng(seed)
    keys = []
    for start in range(0, m, chunk):
        cnt = min(chunk, m - start)
        u = np.zeros(cnt, dtype=np.int64)
        v = np.zeros(cnt, dtype=np.int64)
        for lvl in range(scale):
            r = rng.random(cnt)
            bit_u = r >= a + b            # quadrants c, d -> lower half (row bit)
            bit_v = ((r >= a) & (r < a + b)) | (r >= a + b + c)   # quadrants b, d -> right half
            u |= bit_u.astype(np.int64) << lvl
            v |= bit_v.astype(np.int64) << lvl
        lo = np.minimum(u, v)
        hi = np.maximum(u, v)
        keep = lo != hi
        keys.append(np.unique(lo[keep] * n + hi[keep]))
    key = np.unique(np.concatenate(keys))
    return key // n, key % n


def rmat_laplacian_device(scale: int, edge_factor: int = 16, abcd=(0.57, 0.19, 0.19, 0.05), seed: int = 2,
                          device=None, chunk: int = 1 << 26, relabel_seed=None):
    """The R-MAT normalised Laplacian I - D^-1/2 W D^-1/2 (configuration 4),
    generated and assembled on the GPU with torch.

    Same construction as rmat_edges + normalized_laplacian (Chakrabarti, Zhan,
    Faloutsos 2004: every edge picks one quadrant (a, b, c, d) per level;
    symmetrised, duplicates and self-loops dropped, unit weights, isolated
    vertices get L_ii = 0), drawn from the torch CUDA generator seeded with
    `seed`, so the graph differs from the numpy one of the same seed.
    relabel_seed (not None) renumbers the vertices by a seeded random
    permutation (a symmetric permutation: same graph, same spectrum), so that
    equal row blocks carry about the same number of nonzeros: every level of
    the R-MAT recursion biases one index bit, so contiguous blocks of the
    original numbering are unbalanced (76 % / 24 % of the nonzeros for two
    halves at a = 0.57).  info["perm"] holds the permutation (old -> new).
    Returns (n, rowptr int32, col int32, val float64) device tensors (rows
    sorted by column, the diagonal stored for every row) and an info dict."""
    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    a, b, c, _ = abcd
    n = 1 << scale
    m = edge_factor * n
    g = torch.Generator(device=dev).manual_seed(seed)
    keys = []
    for start in range(0, m, chunk):
        cnt = min(chunk, m - start)
        u = torch.zeros(cnt, dtype=torch.int64, device=dev)
        v = torch.zeros(cnt, dtype=torch.int64, device=dev)
        for lvl in range(scale):
            r = torch.rand(cnt, generator=g, device=dev, dtype=torch.float64)
            u |= (r >= a + b).to(torch.int64) << lvl
            v |= (((r >= a) & (r < a + b)) | (r >= a + b + c)).to(torch.int64) << lvl
        lo, hi = torch.minimum(u, v), torch.maximum(u, v)
        keep = lo != hi
        keys.append(torch.unique(lo[keep] * n + hi[keep]))
        del u, v, lo, hi, keep
    key = torch.unique(torch.cat(keys))
    del keys
    src, dst = key // n, key % n
    del key
    perm = None
    if relabel_seed is not None:
        pg = torch.Generator(device=dev).manual_seed(int(relabel_seed))
        perm = torch.randperm(n, generator=pg, device=dev)
        src, dst = perm[src], perm[dst]
    deg = torch.bincount(src, minlength=n) + torch.bincount(dst, minlength=n)
    dinv = torch.where(deg > 0, deg.to(torch.float64).clamp(min=1).rsqrt(), torch.zeros((), dtype=torch.float64,
                                                                                           device=dev))
    w = -(dinv[src] * dinv[dst])
    diag = torch.arange(n, device=dev, dtype=torch.int64)
    rows = torch.cat([src, dst, diag])
    cols = torch.cat([dst, src, diag])
    vals = torch.cat([w, w, (deg > 0).to(torch.float64)])
    edges = int(src.numel())
    del src, dst, w
    order = torch.argsort(rows * n + cols)
    col = cols[order].to(torch.int32)
    val = vals[order]
    counts = torch.bincount(rows, minlength=n)
    del rows, cols, vals, order
    rowptr = torch.zeros(n + 1, dtype=torch.int32, device=dev)
    rowptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    info = {"n": n, "edges": edges, "nnz": int(col.numel()), "max_degree": int(deg.max()),
            "isolated": int((deg == 0).sum()), "scale": scale, "edge_factor": edge_factor, "seed": seed,
            "relabel_seed": relabel_seed, "perm": perm}
    return n, rowptr, col, val, info


def normalized_laplacian(n: int, src, dst, dtype=np.float64) -> sp.csr_matrix:
    """I - D^-1/2 W D^-1/2 for unit edge weights (isolated vertices: L_ii = 0)."""
    w = np.ones(src.shape[0], dtype=np.float64)
    A = sp.csr_matrix((np.concatenate([w, w]), (np.concatenate([src, dst]), np.concatenate([dst, src]))),
                      shape=(n, n))
    deg = np.asarray(A.sum(axis=1)).ravel()
    dinv = np.zeros(n)
    nz = deg > 0
    dinv[nz] = 1.0 / np.sqrt(deg[nz])
    S = sp.diags(dinv) @ A @ sp.diags(dinv)
    L = (sp.diags(nz.astype(np.float64)) - S).tocsr().astype(dtype)
    L.sum_duplicates()
    L.sort_indices()
    return L
