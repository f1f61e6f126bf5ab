"""GPU kNN search and kNN Laplacian assembly (gpu_eigsh.graph -> lg_knn,
lg_knn_laplacian_rows / _fill) against the oracle restatements of the
reference's builders (oracle/graph.py: src/main.cu:30-107 and
benchmark/generate_large_laplacian.py, the latter pinned to the script's own
output in tests/golden/graph_generator.npz).

Neighbour lists are integer work and distances are contraction-free fp64
sums: both are compared bit for bit.  Laplacian values go through exp(),
whose last bit may differ between the device and the host library: 1e-14
relative, structure exact."""
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden" / "graph_generator.npz"


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    return torch


def _lattice(m, dim):
    g = np.stack(np.meshgrid(*[np.arange(m)] * dim, indexing="ij"), -1).reshape(-1, dim)
    return g.astype(np.float64)


CLOUDS = {
    "u1": lambda: np.random.default_rng(1).uniform(size=(700, 1)),
    "u2": lambda: np.random.default_rng(2).uniform(size=(1500, 2)),
    "u3": lambda: np.random.default_rng(3).uniform(size=(1200, 3)),
    "lattice2": lambda: _lattice(17, 2),
    "lattice3_dup": lambda: np.vstack([_lattice(6, 3), _lattice(6, 3)[::7]]),
    "elongated3": lambda: np.random.default_rng(4).normal(size=(900, 3)) * np.array([100.0, 1.0, 0.01]),
    "clusters2": lambda: np.vstack([np.random.default_rng(5).normal(size=(600, 2)) * 1e-3,
                                    np.random.default_rng(6).normal(size=(200, 2)) + 50.0]),
    "flat2": lambda: np.c_[np.random.default_rng(7).uniform(size=500), np.zeros(500)],
    "u5": lambda: np.random.default_rng(8).uniform(size=(800, 5)),
    "u10": lambda: np.random.default_rng(9).uniform(size=(900, 10)),
    "u20": lambda: np.random.default_rng(10).normal(size=(500, 20)),
}


@pytest.mark.parametrize("cloud", sorted(CLOUDS))
@pytest.mark.parametrize("k", [1, 7, 16, 40])
def test_knn_matches_oracle_bit_for_bit(torch_cuda, cloud, k):
    from gpu_eigsh.graph import knn
    from oracle.graph import knn_bruteforce

    pts = CLOUDS[cloud]()
    ref_i, ref_d = knn_bruteforce(pts, k)
    methods = ["auto", "brute"] + (["cells"] if pts.shape[1] <= 3 else [])
    for m in methods:
        idx, d2 = knn(pts, k, method=m)
        assert np.array_equal(idx.cpu().numpy(), ref_i), (cloud, k, m)
        assert np.array_equal(d2.cpu().numpy(), ref_d), (cloud, k, m)


def test_knn_max_k_and_tiny_n(torch_cuda):
    from gpu_eigsh.graph import knn
    from oracle.graph import knn_bruteforce

    pts = np.random.default_rng(11).uniform(size=(65, 2))
    for k in (63, 64):
        idx, d2 = knn(pts, k)
        ri, rd = knn_bruteforce(pts, k)
        assert np.array_equal(idx.cpu().numpy(), ri) and np.array_equal(d2.cpu().numpy(), rd)
    idx, _ = knn(np.array([[0.0], [1.0]]), 1)
    assert idx.cpu().numpy().ravel().tolist() == [1, 0]


def test_knn_rejects_bad_input(torch_cuda):
    from gpu_eigsh.graph import knn

    pts = np.random.default_rng(12).uniform(size=(50, 3))
    with pytest.raises(ValueError):
        knn(pts, 50)
    with pytest.raises(RuntimeError, match="min\\(64"):
        knn(np.random.default_rng(0).uniform(size=(100, 2)), 65)
    bad = pts.copy()
    bad[7, 1] = np.nan
    with pytest.raises(RuntimeError, match="finite"):
        knn(bad, 4)
    with pytest.raises(RuntimeError, match="dim <= 3"):
        knn(np.random.default_rng(0).uniform(size=(40, 4)), 3, method="cells")


def _csr(torch, rp, ci, va, n):
    import scipy.sparse as sp

    return sp.csr_matrix((va.cpu().numpy(), ci.cpu().numpy(), rp.cpu().numpy()), shape=(n, n))


@pytest.mark.parametrize("cloud,k,bw", [("u2", 10, 0.05), ("u3", 8, 0.1), ("u10", 15, 0.3),
                                        ("lattice3_dup", 6, 1.0), ("clusters2", 12, 0.5)])
def test_laplacian_matches_driver_oracle(torch_cuda, cloud, k, bw):
    from gpu_eigsh.graph import knn_laplacian
    from oracle.graph import driver_laplacian, knn_bruteforce

    pts = CLOUDS[cloud]()
    n = pts.shape[0]
    rp, ci, va = knn_laplacian(pts, k, bw)
    ref_rp, ref_ci, ref_va = driver_laplacian(*knn_bruteforce(pts, k), bw)
    assert np.array_equal(rp.cpu().numpy(), ref_rp) and np.array_equal(ci.cpu().numpy(), ref_ci)
    np.testing.assert_allclose(va.cpu().numpy(), ref_va, rtol=1e-14, atol=0)
    L = _csr(torch_cuda, rp, ci, va, n)
    assert abs(L - L.T).max() == 0.0                      # exactly symmetric
    assert np.abs(L @ np.ones(n)).max() <= 1e-13 * k      # rows sum to zero


def test_generator_matrices_match_reference_output(torch_cuda):
    import scipy.sparse as sp

    from gpu_eigsh.graph import generate_knn_laplacian

    z = np.load(GOLD)
    for c in range(int(z["ncases"])):
        n, dim, k, bw, seed = z[f"c{c}_args"]
        L = generate_knn_laplacian(int(n), int(dim), int(k), float(bw), int(seed))
        R = sp.csr_matrix((z[f"c{c}_data"], z[f"c{c}_indices"], z[f"c{c}_indptr"]), shape=(int(n), int(n)))
        assert np.array_equal(L.indptr, R.indptr) and np.array_equal(L.indices, R.indices)
        np.testing.assert_allclose(L.data, R.data, rtol=1e-13, atol=0)


def test_laplacian_rejects_bad_lists(torch_cuda):
    torch = torch_cuda
    from gpu_eigsh.graph import laplacian_from_knn

    idx = torch.tensor([[1, 2], [0, 2], [0, 1], [1, 1]], dtype=torch.int64, device="cuda")
    d2 = torch.ones((4, 2), dtype=torch.float64, device="cuda")
    with pytest.raises(RuntimeError, match="distinct"):
        laplacian_from_knn(idx, d2, 1.0)          # row 3 lists 1 twice
    idx[3] = torch.tensor([3, 0])
    with pytest.raises(RuntimeError, match="distinct"):
        laplacian_from_knn(idx, d2, 1.0)          # self edge
    idx[3] = torch.tensor([0, 9])
    with pytest.raises(RuntimeError, match="distinct"):
        laplacian_from_knn(idx, d2, 1.0)          # out of range


def _sample_rows_exact(torch, P, rows, k):
    """Exact neighbour lists of a few rows by torch on the device: squared
    differences summed in coordinate order by separate elementwise kernels
    (no contraction), stable sort on the distance over ascending indices."""
    out_i, out_d = [], []
    for r in rows:
        s = torch.zeros(P.shape[0], dtype=torch.float64, device=P.device)
        for d in range(P.shape[1]):
            t = P[:, d] - P[r, d]
            s = s + t * t
        s[r] = float("inf")
        v, o = torch.sort(s, stable=True)
        out_i.append(o[:k])
        out_d.append(v[:k])
    return torch.stack(out_i), torch.stack(out_d)


@pytest.mark.parametrize("n,dim,k", [(1_000_000, 2, 10), (1_000_000, 3, 15), (100_000, 10, 15)])
def test_knn_full_size_sampled_rows(torch_cuda, n, dim, k):
    """Full-size clouds: 64 random rows compared with an exact device
    computation; every list ascending; the graph Laplacian symmetric with
    zero row sums."""
    torch = torch_cuda
    from gpu_eigsh.graph import knn, laplacian_from_knn

    P = torch.from_numpy(np.random.default_rng(n + dim).uniform(size=(n, dim))).cuda()
    idx, d2 = knn(P, k)
    rows = torch.from_numpy(np.random.default_rng(1).choice(n, 64, replace=False)).cuda()
    ri, rd = _sample_rows_exact(torch, P, rows.tolist(), k)
    assert torch.equal(idx[rows], ri) and torch.equal(d2[rows], rd)
    assert bool((d2[:, 1:] >= d2[:, :-1]).all())
    rp, ci, va = laplacian_from_knn(idx, d2, 0.3)
    rs = torch.zeros(n, dtype=torch.float64, device="cuda").index_add_(
        0, torch.repeat_interleave(torch.arange(n, device="cuda"), (rp[1:] - rp[:-1]).long()), va)
    assert float(rs.abs().max()) <= 1e-12
    assert int(rp[-1]) >= n * (k + 1)
