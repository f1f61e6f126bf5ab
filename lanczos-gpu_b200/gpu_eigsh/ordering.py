"""Row orderings of symmetric sparse matrices for locality.

``bfs_order`` numbers the vertices of the graph of a symmetric CSR by
breadth-first level from a pseudo-peripheral vertex (two sweeps of
lg_graph_bfs_levels on the GPU), ties broken by the old index; ``cm_order``
(Cuthill-McKee, on the host) also orders each level by the vertices that
found it.  Rows that are neighbours in the graph get nearby numbers, so

* the sparse products of the SLQ operator gather from rows that a CTA's
  neighbours also read (L2 hits), and
* a contiguous row partition over several GPUs has small halos (the rows a
  rank's columns name outside its own block lie in the adjacent levels).

``degree_order`` sorts the vertices by descending degree instead, for
power-law graphs (R-MAT, web and social graphs) that have no bandwidth to
reduce: most column indices name a few hub vertices, and numbering those first
packs the entries of the vector that the sparse product gathers most often into
a few cache sectors that stay in L2.  With ``parts`` > 1 the sorted vertices are
dealt round-robin to the row blocks of a partition, so every GPU gets the same
share of hubs and of nonzeros, and inside each block the hubs come first.

``permute_symmetric`` applies the numbering: P A P^T, which has the same
eigenvalues; eigenvectors come back with ``x_old = x_new[pos]``.

The reference keeps the caller's order (python/gpu_eigsh/imgp.py builds its
operator on the caller's vertex numbering; src/ has no reordering).
"""
from __future__ import annotations

import torch

from . import _native

__all__ = ["bfs_levels", "bfs_order", "cm_order", "degree_order", "permute_symmetric"]


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def bfs_levels(rowptr: torch.Tensor, col: torch.Tensor, start: int) -> torch.Tensor:
    """Hop distance of every vertex from `start` (-1 where unreachable) in the
    graph of a CSR with every edge stored both ways (int32 device tensors)."""
    n = rowptr.numel() - 1
    dev = rowptr.device
    level = torch.empty(n, dtype=torch.int32, device=dev)
    work = torch.empty(2 * n + 2, dtype=torch.int32, device=dev)
    rounds = _native.C.c_int(0)
    _native.check(_native.lib.lg_graph_bfs_levels(n, rowptr.data_ptr(), col.data_ptr(), int(start), level.data_ptr(),
                                                  work.data_ptr(), _native.C.byref(rounds), _stream(dev)))
    return level


def bfs_order(rowptr: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """perm (int64, device): perm[new] = old, vertices sorted by (BFS level
    from a pseudo-peripheral vertex, old index); unreachable vertices last."""
    n = rowptr.numel() - 1
    level = bfs_levels(rowptr, col, 0)
    start = int(torch.argmax(level))             # a farthest vertex from 0
    level = bfs_levels(rowptr, col, start).to(torch.int64)
    level = torch.where(level < 0, torch.full_like(level, n), level)
    return torch.argsort(level * n + torch.arange(n, device=rowptr.device))


def cm_order(rowptr: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """perm (int64, on rowptr's device): the Cuthill-McKee order of the graph
    of a symmetric CSR (lg_graph_cm_order, computed on the host): BFS levels
    as bfs_order, and inside a level the order of the vertices that found
    them, so that consecutive rows also gather neighbouring rows."""
    import numpy as np

    n = rowptr.numel() - 1
    rp = np.ascontiguousarray(rowptr.detach().cpu().numpy(), dtype=np.int32)
    ci = np.ascontiguousarray(col.detach().cpu().numpy(), dtype=np.int32)
    perm = np.empty(n, dtype=np.int32)
    PI = _native.C.POINTER(_native.C.c_int)
    _native.check(_native.lib.lg_graph_cm_order(n, rp.ctypes.data_as(PI), ci.ctypes.data_as(PI),
                                                perm.ctypes.data_as(PI)))
    return torch.from_numpy(perm.astype(np.int64)).to(rowptr.device)


def degree_order(rowptr: torch.Tensor, parts: int = 1) -> torch.Tensor:
    """perm (int64, on rowptr's device): perm[new] = old.  The vertices sorted
    by (descending degree, index); with ``parts`` > 1, dealt in that order to
    the row blocks of ``distributed.partition_rows(n, parts, r)`` (vertex i of
    the sorted list to block i mod parts while every block has room), each
    block keeping the dealt order.  parts=1 is the order that
    LG_PLAN_REORDER_DEGREE applies inside a plan."""
    n = rowptr.numel() - 1
    dev = rowptr.device
    rp = rowptr.to(torch.int64)
    deg = rp[1:] - rp[:-1]
    # stable sort on the key (max_degree - degree) * n + index: ties by index
    key = (deg.max() - deg) * n + torch.arange(n, device=dev) if n > 0 else deg
    srt = torch.argsort(key)
    if parts <= 1 or n == 0:
        return srt
    from .distributed import partition_rows

    bounds = [partition_rows(n, parts, r) for r in range(parts)]
    nb = max(b - a for a, b in bounds)
    slot = torch.arange(nb, device=dev).view(-1, 1)
    start = torch.tensor([a for a, _ in bounds], device=dev).view(1, -1)
    size = torch.tensor([b - a for a, b in bounds], device=dev).view(1, -1)
    target = (start + slot).masked_select(slot < size)   # slot-major: block 0, 1, ... of slot 0, then slot 1, ...
    perm = torch.empty_like(srt)
    perm[target] = srt
    return perm


def permute_symmetric(rowptr: torch.Tensor, col: torch.Tensor, val: torch.Tensor, perm: torch.Tensor,
                      return_order: bool = False):
    """P A P^T of a CSR (row i of the result = row perm[i] of A, columns
    renumbered by pos = perm^-1 and sorted).  Returns (rowptr int32, col
    int32, val, pos int64) on the device of the inputs, and with return_order
    also `order` (int64): entry j of the result is entry order[j] of A."""
    n = rowptr.numel() - 1
    dev = rowptr.device
    perm = perm.to(dev, torch.int64)
    pos = torch.empty_like(perm)
    pos[perm] = torch.arange(n, device=dev)
    rp = rowptr.to(torch.int64)
    counts = rp[1:] - rp[:-1]
    rows_old = torch.repeat_interleave(torch.arange(n, device=dev), counts)
    r_new = pos[rows_old]
    c_new = pos[col.to(torch.int64)]
    order = torch.argsort(r_new * n + c_new)
    new_counts = counts[perm]
    out_rp = torch.zeros(n + 1, dtype=torch.int32, device=dev)
    out_rp[1:] = torch.cumsum(new_counts, 0).to(torch.int32)
    out = (out_rp, c_new[order].to(torch.int32).contiguous(), val[order].contiguous(), pos)
    return out + (order,) if return_order else out
