"""CPU (gloo, world sizes 2 and 3): the halo plan of the row-partitioned eigsh.

Every rank runs the library's host planning (lg_halo_recv_list, then
lg_halo_send_plan on the count matrix all-reduced over gloo), hands its
receive positions to their owners (the owners' send lists), packs its own
rows at those positions, and unpacks what it receives at the same global
positions; every column the rank's CSR names must then hold the entry of the
dense vector (the all-gather the halo replaces).  The ranks must agree on the
exchange mode, and one case gives a rank no remote columns at all.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import scipy.sparse as sp
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _matrix(case, n):
    rng = np.random.default_rng(3)
    if case == "banded":       # a thin boundary between neighbouring blocks: halo mode
        off = rng.integers(1, 40, size=6 * n)
        rows = rng.integers(0, n, size=6 * n)
        cols = np.clip(rows + off, 0, n - 1)
    elif case == "random":     # every block reads from every block: all-gather mode
        rows = rng.integers(0, n, size=8 * n)
        cols = rng.integers(0, n, size=8 * n)
    else:                      # "isolated": the last rank's rows form their own component
        nb = _block(n, 3)
        head = 2 * nb
        rows = rng.integers(0, head, size=6 * n)
        cols = rng.integers(0, head, size=6 * n)
        r2 = rng.integers(head, n, size=n)
        c2 = rng.integers(head, n, size=n)
        rows, cols = np.concatenate([rows, r2]), np.concatenate([cols, c2])
    A = sp.csr_matrix((np.ones(rows.shape[0]), (rows, cols)), shape=(n, n))
    A = (A + A.T + sp.identity(n)).tocsr()
    A.sum_duplicates()
    A.sort_indices()
    return A


def _block(n, world):
    from gpu_eigsh import _native

    return _native.lib.lg_partition_block(n, world)


def _worker(rank, world, port, case, n, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gpu_eigsh import _native

        lib = _native.lib
        A = _matrix(case, n)
        nb = _block(n, world)
        r0, r1 = min(rank * nb, n), min((rank + 1) * nb, n)
        col = np.ascontiguousarray(A.indices[A.indptr[r0]:A.indptr[r1]], dtype=np.int32)
        PI = C.POINTER(C.c_int)
        cnt = np.zeros(world, dtype=np.int64)
        total = C.c_longlong(0)
        # first call sizes the list (capacity 0), second fills it
        rc = lib.lg_halo_recv_list(n, world, rank, col.shape[0], col.ctypes.data_as(PI), None, 0,
                                   cnt.ctypes.data_as(C.POINTER(C.c_longlong)), C.byref(total))
        assert rc == (_native.LG_ERR_INVALID if total.value > 0 else 0)
        recv = np.zeros(max(total.value, 1), dtype=np.int32)
        assert lib.lg_halo_recv_list(n, world, rank, col.shape[0], col.ctypes.data_as(PI), recv.ctypes.data_as(PI),
                                     recv.shape[0], cnt.ctypes.data_as(C.POINTER(C.c_longlong)),
                                     C.byref(total)) == 0
        recv = recv[:total.value]
        # receive list: only other ranks' rows, grouped by owner, ascending
        owners = recv // nb
        assert np.all(owners != rank) and np.all(np.diff(owners) >= 0)
        for o in range(world):
            seg = recv[owners == o]
            assert np.all(np.diff(seg) > 0) and seg.shape[0] == cnt[o]
        # exactly the remote columns this rank's CSR names
        remote = np.unique(col[(col < r0) | (col >= r1)])
        assert np.array_equal(np.sort(recv), remote)

        M = torch.zeros(world * world, dtype=torch.float64)
        M[rank * world:(rank + 1) * world] = torch.from_numpy(cnt.astype(np.float64))
        dist.all_reduce(M)
        send_cnt = np.zeros(world, dtype=np.int64)
        mode = C.c_int(-1)
        assert lib.lg_halo_send_plan(n, world, rank, M.numpy().ctypes.data_as(C.POINTER(C.c_double)),
                                     send_cnt.ctypes.data_as(C.POINTER(C.c_longlong)), C.byref(mode)) == 0

        # owners learn the positions (the grouped exchange of the plan)
        lists = [None] * world
        dist.all_gather_object(lists, recv.tolist())
        send_idx = {p: [c for c in lists[p] if r0 <= c < r1] for p in range(world) if p != rank}
        for p, idx in send_idx.items():
            assert len(idx) == send_cnt[p]
        # pack my rows, exchange, unpack at the global positions
        x = np.sin(np.arange(n) * 0.37) + 2.0          # the dense vector
        full = np.full(world * nb, np.nan)
        full[r0:r1] = x[r0:r1]
        packed = [None] * world
        dist.all_gather_object(packed, {p: x[idx].tolist() for p, idx in send_idx.items()})
        got = 0
        for q in range(world):
            if q == rank:
                continue
            vals = np.asarray(packed[q].get(rank, []))
            pos = recv[owners == q]
            assert vals.shape[0] == pos.shape[0]
            full[pos] = vals
            got += vals.shape[0]
        assert got == total.value
        # every column this rank's product reads holds the dense entry
        assert np.array_equal(full[col], x[col])
        out[rank] = torch.tensor([mode.value, total.value, int(send_cnt.sum())], dtype=torch.float64)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case, world", [("banded", 2), ("banded", 3), ("random", 2), ("random", 3),
                                         ("isolated", 3)])
def test_halo_plan_reaches_every_named_column(case, world):
    n = 3000
    out = torch.zeros(world, 3, dtype=torch.float64).share_memory_()
    mp.spawn(_worker, args=(world, _free_port(), case, n, out), nprocs=world, join=True)
    modes = out[:, 0].tolist()
    assert len(set(modes)) == 1, "ranks chose different exchange modes"
    if case == "banded":
        assert modes[0] == 2      # LG_EXCHANGE_HALO
    if case == "random":
        assert modes[0] == 1      # LG_EXCHANGE_ALLGATHER
    if case == "isolated":
        assert out[world - 1, 1] == 0 and out[world - 1, 2] == 0, "the isolated rank has no halo"
    # every row received was sent
    assert out[:, 1].sum() == out[:, 2].sum()
