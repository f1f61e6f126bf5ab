"""GPU (2+ devices): the row-partitioned eigsh equals the single-GPU solve.

Two ranks (processes, one GPU each) split the rows of a kNN graph
Laplacian (in the generator's order, and renumbered by BFS level so that the
halos are small: run with the halo exchange and, forced, with the
all-gather) and of an R-MAT normalised Laplacian (configuration 4's family,
with rows longer than the row kernels' cut; in the generator's order, and
sorted by degree with the hubs dealt to the two blocks), through the peer-memory
transport (reductions and exchanges as kernels storing into the other rank's
memory) and, for two cases, through NCCL.  Every rank must report the same
eigenvalues, equal to the single-GPU plan's and to scipy ARPACK's at 1e-10, and the assembled
eigenvector rows must satisfy ||A v - lambda v|| <= tol ||A||.  Skipped with
fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest
import scipy.sparse as sp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _matrix(case):
    from gpu_eigsh import synthetic as syn

    if case.startswith("knn"):
        L, _ = syn.knn_laplacian(60000, k=10, seed=4)
        if case != "knn":
            import torch

            from gpu_eigsh.ordering import bfs_order, permute_symmetric

            dev = torch.device("cuda", torch.cuda.current_device())
            rp = torch.from_numpy(L.indptr.astype(np.int32)).to(dev)
            ci = torch.from_numpy(L.indices.astype(np.int32)).to(dev)
            va = torch.from_numpy(L.data).to(dev)
            rp2, ci2, va2, _ = permute_symmetric(rp, ci, va, bfs_order(rp, ci))
            L = sp.csr_matrix((va2.cpu().numpy(), ci2.cpu().numpy(), rp2.cpu().numpy()), shape=L.shape)
        return L, dict(k=10, which="LA", ncv=30, tol=1e-10), False
    import torch

    n, rp, col, val, _ = syn.rmat_laplacian_device(15, device="cpu")
    if case == "rmat_degree":
        # hubs first, dealt round-robin to the two row blocks
        from gpu_eigsh.ordering import degree_order, permute_symmetric

        rp, col, val, _ = permute_symmetric(rp, col, val, degree_order(rp, 2))
    L = sp.csr_matrix((val.numpy(), col.numpy(), rp.numpy()), shape=(n, n))
    return L, dict(k=12, which="LA", ncv=40, tol=1e-10), False


def _worker(rank, world, port, case, out_w, out_y):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from gpu_eigsh.distributed import Communicator, PartitionedEigsh, partition_rows

    comm = Communicator()
    try:
        L, kw, _ = _matrix(case)
        n = L.shape[0]
        r0, r1 = partition_rows(n, world, rank)
        a, b = L.indptr[r0], L.indptr[r1]
        dev = torch.device("cuda", rank)
        rp = torch.from_numpy((L.indptr[r0:r1 + 1] - a).astype(np.int32)).to(dev)
        col = torch.from_numpy(L.indices[a:b].astype(np.int32)).to(dev)
        val = torch.from_numpy(L.data[a:b].astype(np.float64)).to(dev)
        v0 = np.random.default_rng(0).standard_normal(n)
        forced = {"knn_bfs_allgather": "allgather"}.get(case, "auto")
        transport = "nccl" if case.endswith("_nccl") else "auto"
        pe = PartitionedEigsh(comm, n, rp, col, val, max_ncv=kw["ncv"], exchange=forced, transport=transport)
        # one GPU per rank: the reductions and exchanges go through the
        # peer-memory kernels unless NCCL is asked for
        assert pe.transport == ("nccl" if transport == "nccl" else "peer"), pe.transport
        k = kw.pop("k")
        w, Y = pe.solve(k, v0[r0:r1], **kw)
        torch.cuda.synchronize()
        out_w[rank, :k] = torch.from_numpy(np.asarray(w))
        out_y[r0:r1, :k] = Y.cpu()
        mode, recv_rows, send_rows = pe.exchange_info
        pe.close()
        # the BFS numbering leaves a thin boundary between the two row blocks
        if case in ("knn_bfs", "knn_bfs_nccl"):
            assert mode == "halo" and 0 < recv_rows < (r1 - r0) // 4, (mode, recv_rows)
        if case == "knn_bfs_allgather":
            assert mode == "allgather"
        if case.startswith("rmat"):
            assert mode == "allgather", (mode, recv_rows)
    finally:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["knn", "knn_bfs", "knn_bfs_allgather", "rmat", "knn_bfs_nccl", "rmat_nccl",
                                  "rmat_degree"])
def test_partitioned_equals_single_gpu(case):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import gpu_eigsh

    world = 2
    L, kw, _ = _matrix(case)
    n, k = L.shape[0], kw["k"]
    out_w = torch.zeros(world, k, dtype=torch.float64).share_memory_()
    out_y = torch.zeros(n, k, dtype=torch.float64).share_memory_()
    mp.spawn(_worker, args=(world, _free_port(), case, out_w, out_y), nprocs=world, join=True)
    assert torch.equal(out_w[0], out_w[1]), "ranks disagree on the eigenvalues"
    v0 = np.random.default_rng(0).standard_normal(n)
    ref = gpu_eigsh.gpu_eigsh(L, v0=v0, return_eigenvectors=False, **kw)
    w = out_w[0].numpy()
    assert np.max(np.abs(w - np.sort(ref)) / np.maximum(np.abs(ref), 1e-300)) < 1e-10
    # and the ground truth itself: scipy's ARPACK with the same arguments
    from oracle.irlm import arpack_eigsh

    from _parity import anorm1, eig_rel_err

    kw_a = {key: kw[key] for key in ("which", "ncv", "tol")}
    ws, _ = arpack_eigsh(L, k, v0=v0, **kw_a)
    assert eig_rel_err(w, ws, anorm1(L)) < 1e-10
    Y = out_y.numpy()
    res = np.linalg.norm(L @ Y - Y * w, axis=0).max()
    assert res <= kw["tol"] * abs(L).sum(axis=1).max()


def _timeout_worker(rank, world, port, out):
    """Rank 1 builds the plan (a collective) but never solves with it: rank
    0's first peer wait finds no flag and gives up after LG_PEER_WAIT_MS.
    Then both ranks build a new plan and solve normally on the same
    contexts."""
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LG_PEER_WAIT_MS="300",
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    import gpu_eigsh
    from gpu_eigsh import _native
    from gpu_eigsh.distributed import Communicator, PartitionedEigsh, partition_rows

    comm = Communicator()
    try:
        L, kw, _ = _matrix("knn_bfs")
        n = L.shape[0]
        r0, r1 = partition_rows(n, world, rank)
        a, b = L.indptr[r0], L.indptr[r1]
        dev = torch.device("cuda", rank)

        def plan():
            rp = torch.from_numpy((L.indptr[r0:r1 + 1] - a).astype(np.int32)).to(dev)
            col = torch.from_numpy(L.indices[a:b].astype(np.int32)).to(dev)
            val = torch.from_numpy(L.data[a:b].astype(np.float64)).to(dev)
            return PartitionedEigsh(comm, n, rp, col, val, max_ncv=kw["ncv"]), (rp, col, val)

        v0 = np.random.default_rng(0).standard_normal(n)[r0:r1]
        pe, keep = plan()
        assert pe.transport == "peer"
        status = 0
        if rank == 0:
            with pytest.raises(gpu_eigsh.LanczosError) as ei:
                pe.solve(kw["k"], v0, which="LA", ncv=kw["ncv"], tol=kw["tol"])
            status = ei.value.status
        torch.cuda.synchronize()
        pe.close()
        dist.barrier()
        pe, keep = plan()
        w, _ = pe.solve(kw["k"], v0, which="LA", ncv=kw["ncv"], tol=kw["tol"])
        torch.cuda.synchronize()
        pe.close()
        out[rank, 0] = float(status)
        out[rank, 1] = float(w[-1])
        assert status == (_native.LG_ERR_TIMEOUT if rank == 0 else 0)
    finally:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def test_peer_wait_gives_up_when_a_rank_is_absent():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = torch.zeros(2, 2, dtype=torch.float64).share_memory_()
    mp.spawn(_timeout_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    from gpu_eigsh import _native

    assert out[0, 0] == _native.LG_ERR_TIMEOUT and out[1, 0] == 0
    assert out[0, 1] == out[1, 1] and out[0, 1] > 0
