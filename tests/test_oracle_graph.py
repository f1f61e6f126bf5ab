"""The graph-builder oracle (oracle/graph.py) pinned to the reference:
the generator restatement reproduces the matrices the reference's own
benchmark/generate_large_laplacian.py wrote (tests/golden/graph_generator.npz),
and the driver restatement (src/main.cu:30-107) agrees with it on the same
points."""
from pathlib import Path

import numpy as np
import scipy.sparse as sp

from oracle import graph as G

GOLD = Path(__file__).resolve().parent / "golden" / "graph_generator.npz"


def _cases():
    z = np.load(GOLD)
    for c in range(int(z["ncases"])):
        n, dim, k, bw, seed = z[f"c{c}_args"]
        L = sp.csr_matrix((z[f"c{c}_data"], z[f"c{c}_indices"], z[f"c{c}_indptr"]), shape=(int(n), int(n)))
        yield (int(n), int(dim), int(k), float(bw), int(seed)), L


def _same(L, M, rtol):
    L, M = sp.csr_matrix(L), sp.csr_matrix(M)
    assert L.shape == M.shape
    assert np.array_equal(L.indptr, M.indptr) and np.array_equal(L.indices, M.indices)
    np.testing.assert_allclose(L.data, M.data, rtol=rtol, atol=0)


def test_generator_restatement_matches_reference_output():
    for (n, dim, k, bw, seed), L in _cases():
        _same(G.generator_laplacian(n, dim, k, bw, seed), L, 1e-15)


def test_driver_restatement_matches_generator():
    for (n, dim, k, bw, seed), L in _cases():
        pts = G.generator_points(n, dim, seed)
        idx, d2 = G.knn_bruteforce(pts, k)
        rp, ci, va = G.driver_laplacian(idx, d2, bw)
        _same(sp.csr_matrix((va, ci, rp), shape=(n, n)), L, 1e-13)


def test_bruteforce_matches_ckdtree_and_orders_ties_by_index():
    from scipy.spatial import cKDTree

    pts = G.generator_points(300, 3, 5)
    idx, d2 = G.knn_bruteforce(pts, 9)
    dist, ind = cKDTree(pts).query(pts, k=10)
    assert np.array_equal(idx, ind[:, 1:])
    np.testing.assert_allclose(d2, dist[:, 1:] ** 2, rtol=1e-14)
    # a lattice: many equal distances, broken by the smaller index
    lat = np.array([[x, y] for x in range(5) for y in range(5)], dtype=np.float64)
    idx, d2 = G.knn_bruteforce(lat, 4)
    assert list(idx[12]) == [7, 11, 13, 17] and list(d2[12]) == [1.0] * 4
    assert list(idx[0]) == [1, 5, 6, 2]
