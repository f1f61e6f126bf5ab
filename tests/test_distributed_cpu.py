"""CPU (gloo, world size 2): probe-sharded SLQ combines to the single-process
estimate.

The sharding wrapper (gpu_eigsh.distributed) is engine-agnostic; here each
rank drives it with an engine built on the oracle (the reference's algorithm
on the CPU), so the partition of the probes, the all-reduce of the quadrature
sums and the all-reduce of the parameter gradients are checked without a GPU.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import slq as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _graph(n=150, seed=0):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (700,), generator=g)
    dst = torch.randint(0, n, (700,), generator=g)
    keep = src < dst
    idx = torch.stack([src[keep], dst[keep]])
    d2 = torch.rand(idx.shape[1], generator=g, dtype=torch.float64) + 0.1
    return idx, d2


class OracleEngine:
    """forward/backward of the local probe share, by the oracle."""

    def __init__(self, mv, m, params):
        self.mv, self.m, self.params = mv, m, params

    def forward(self, Z_local, p_total, keep=True):
        pd = tuple(p.detach().clone().requires_grad_(True) for p in self.params)
        with torch.enable_grad():
            local_sum = O._SLQ.apply(self.mv, Z_local, self.m, *pd) * Z_local.shape[1]
        return local_sum.detach(), (local_sum, pd, p_total)

    def backward(self, state, g_out):
        local_sum, pd, p_total = state
        g = torch.autograd.grad(local_sum, pd, grad_outputs=g_out.reshape(()))
        return [x / p_total for x in g]


def _worker(rank, world, port, P, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gpu_eigsh.distributed import sharded_slq

        n = 150
        idx, d2 = _graph(n)
        mv = O.make_precision_matvec(d2, idx, n, 2)
        e = torch.tensor(0.9, dtype=torch.float64, requires_grad=True)
        k = torch.tensor(1.1, dtype=torch.float64, requires_grad=True)
        Z = O.rademacher(n, P, 7, torch.float64)
        ld = sharded_slq(OracleEngine(mv, 12, (e, k)), Z, (e, k))
        ld.backward()
        out[rank] = torch.tensor([float(ld.detach()), float(e.grad), float(k.grad)], dtype=torch.float64)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("P", [6, 7, 1])
def test_probe_sharded_slq_matches_single_process(P):
    world = 2
    out = torch.zeros(world, 3, dtype=torch.float64).share_memory_()
    mp.spawn(_worker, args=(world, _free_port(), P, out), nprocs=world, join=True)
    n = 150
    idx, d2 = _graph(n)
    mv = O.make_precision_matvec(d2, idx, n, 2)
    e = torch.tensor(0.9, dtype=torch.float64, requires_grad=True)
    k = torch.tensor(1.1, dtype=torch.float64, requires_grad=True)
    ld = O.slq_logdet(mv, n, (e, k), m_probes=P, lanczos_m=12, seed=7)
    ld.backward()
    ref = torch.tensor([float(ld.detach()), float(e.grad), float(k.grad)], dtype=torch.float64)
    for r in range(world):
        assert torch.allclose(out[r], ref, rtol=1e-12, atol=0), (r, out[r], ref)


def test_probe_range_partitions():
    from gpu_eigsh.distributed import probe_range

    for P in (1, 7, 64, 130):
        for world in (1, 2, 3, 8):
            cols = []
            for r in range(world):
                c0, c1 = probe_range(P, r, world)
                assert 0 <= c1 - c0 <= P // world + 1
                cols += list(range(c0, c1))
            assert cols == list(range(P))


def test_partition_rows_covers_every_row_once():
    from gpu_eigsh import _native
    from gpu_eigsh.distributed import partition_rows

    for n in (1000, 60000, 1 << 20, 16777216):
        for world in (1, 2, 3, 4, 8):
            nb = _native.lib.lg_partition_block(n, world)
            assert nb % 256 == 0 and nb * world >= n
            rows = []
            for r in range(world):
                r0, r1 = partition_rows(n, world, r)
                assert r0 == min(r * nb, n)
                rows.append((r0, r1))
            assert rows[0][0] == 0 and rows[-1][1] == n
            assert all(rows[i][1] == rows[i + 1][0] for i in range(world - 1))


def test_permute_symmetric_matches_scipy():
    """P A P^T of a CSR (the renumbering applied before a row partition) equals
    scipy's on CPU tensors, with sorted columns."""
    import numpy as np

    from gpu_eigsh import synthetic as syn
    from gpu_eigsh.ordering import permute_symmetric

    L, _ = syn.knn_laplacian(3000, k=6, seed=3)
    perm = torch.from_numpy(np.random.default_rng(1).permutation(L.shape[0]))
    rp, ci, va, pos = permute_symmetric(torch.from_numpy(L.indptr.astype(np.int32)),
                                        torch.from_numpy(L.indices.astype(np.int32)), torch.from_numpy(L.data), perm)
    P = L[perm.numpy()][:, perm.numpy()].tocsr()
    P.sort_indices()
    np.testing.assert_array_equal(rp.numpy(), P.indptr)
    np.testing.assert_array_equal(ci.numpy(), P.indices)
    np.testing.assert_array_equal(va.numpy(), P.data)
    np.testing.assert_array_equal(pos.numpy()[perm.numpy()], np.arange(L.shape[0]))


def test_differentiable_values_bypass_dense_gradient():
    """The values of a torch sparse CSR tensor reach differentiable_eigsh
    without torch's dense n x n gradient of the sparse constructor (checked on
    CPU: the routing only, no eigensolve)."""
    import warnings

    from gpu_eigsh.differentiable import _direct_values

    warnings.filterwarnings("ignore")
    n = 50
    crow = torch.arange(0, n + 1)
    col = torch.arange(n)
    leaf = torch.ones(n, dtype=torch.float64, requires_grad=True)
    vals = leaf * 3.0
    A = torch.sparse_csr_tensor(crow, col, vals, (n, n))
    v = _direct_values(A)
    assert v is vals
    (v * 2.0).sum().backward()
    assert torch.equal(leaf.grad, torch.full((n,), 6.0, dtype=torch.float64))
    B = torch.sparse_csr_tensor(crow, col, torch.ones(n, dtype=torch.float64), (n, n))
    assert torch.equal(_direct_values(B), B.values())


def test_cm_order_is_a_bandwidth_reducing_permutation():
    """lg_graph_cm_order (host code, no GPU): a permutation of every component,
    starting each at a pseudo-peripheral vertex, with a far smaller bandwidth
    than a random numbering of the same kNN graph."""
    import numpy as np

    from gpu_eigsh import synthetic as syn
    from gpu_eigsh.ordering import cm_order, permute_symmetric

    L, _ = syn.knn_laplacian(5000, k=8, seed=2)
    rp = torch.from_numpy(L.indptr.astype(np.int32))
    ci = torch.from_numpy(L.indices.astype(np.int32))
    perm = cm_order(rp, ci)
    assert torch.equal(torch.sort(perm).values, torch.arange(L.shape[0]))
    rp2, ci2, _, _ = permute_symmetric(rp, ci, torch.from_numpy(L.data), perm)
    rows = torch.repeat_interleave(torch.arange(L.shape[0]), (rp2[1:] - rp2[:-1]).long())
    bw_cm = int((rows - ci2.long()).abs().max())
    rows0 = torch.repeat_interleave(torch.arange(L.shape[0]), (rp[1:] - rp[:-1]).long())
    bw_orig = int((rows0 - ci.long()).abs().max())
    assert bw_cm < bw_orig / 10, (bw_cm, bw_orig)
    # two components: both placed, each contiguous
    import scipy.sparse as sp

    B = sp.block_diag([L[:100, :100], L[:50, :50]]).tocsr()
    p2 = cm_order(torch.from_numpy(B.indptr.astype(np.int32)), torch.from_numpy(B.indices.astype(np.int32)))
    assert torch.equal(torch.sort(p2).values, torch.arange(150))


def test_degree_order_sorts_and_deals_hubs():
    """degree_order: descending degree, ties by index (the order
    LG_PLAN_REORDER_DEGREE applies); with parts > 1 the sorted vertices are
    dealt round-robin to the row blocks of partition_rows, so each block gets
    the same share of nonzeros and starts with its hubs."""
    import numpy as np

    from gpu_eigsh import synthetic as syn
    from gpu_eigsh.distributed import partition_rows
    from gpu_eigsh.ordering import degree_order, permute_symmetric

    n, rp, col, val, _ = syn.rmat_laplacian_device(12, device="cpu")
    deg = (rp[1:] - rp[:-1]).long()
    perm = degree_order(rp)
    assert torch.equal(torch.sort(perm).values, torch.arange(n))
    ref = sorted(range(n), key=lambda i: (-int(deg[i]), i))
    assert perm.tolist() == ref
    for parts in (2, 3, 4):
        p = degree_order(rp, parts)
        assert torch.equal(torch.sort(p).values, torch.arange(n))
        rp2, _, _, _ = permute_symmetric(rp, col, val, p)
        nnz_blocks = []
        for r in range(parts):
            r0, r1 = partition_rows(n, parts, r)
            # block r holds sorted positions r, r + parts, ... while it has room
            if n % parts == 0 and r1 - r0 == n // parts:   # equal blocks: a plain round-robin deal
                assert p[r0:r1].tolist() == ref[r::parts]
            d = deg[p[r0:r1]]
            assert torch.all(d[:-1] >= d[1:])
            nnz_blocks.append(int(rp2[r1] - rp2[r0]))
        assert max(nnz_blocks) - min(nnz_blocks) <= 0.02 * max(nnz_blocks) + int(deg.max()), nnz_blocks
