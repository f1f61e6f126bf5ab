"""Multi-GPU paths (one process per GPU, torch.distributed over NCCL).

1. eigsh, row-partitioned (``Communicator``, ``partition_rows``,
   ``PartitionedEigsh``): rank r owns the rows [r*nb, min((r+1)*nb, n)) of the
   matrix (nb = lg_partition_block); before each sparse product the CUDA
   engine exchanges the residual rows other ranks read (a halo exchange of
   grouped NCCL sends and receives when the halos are small, as for a graph
   numbered by ``gpu_eigsh.ordering.bfs_order``; an all-gather otherwise, as
   for power-law graphs), all-reduces one row of partial sums per
   Gram-Schmidt pass with NCCL, and runs the restart logic replicated.  The
   reference runs on one GPU only.

2. Stochastic Lanczos quadrature, probes sharded across ranks:

The probe columns of an SLQ estimate are independent, so N ranks (one process
per GPU, torch.distributed over NCCL) split them: every rank draws the same
probe block (same seed), keeps its contiguous share of the columns, runs the
fused single-GPU engine on it and the ranks combine

  forward   one all-reduce (sum) of the per-rank quadrature sums;
            log det = total / m_probes on every rank;
  backward  one all-reduce (sum) of the per-rank parameter gradients.

The operator (n = 1e6: ~100 MB) is replicated.  Results equal the single-GPU
estimate up to the order of the fp64 sums.  This is the probe sharding of the
reference's batched SLQ (python/gpu_eigsh/funm_torch.py:571-781), which runs on
one device only.

The wrapper works with any engine object offering
    forward(Z_local, p_total, keep) -> (sum of local quadratures (0-d fp64), state)
    backward(state, g_out) -> [gradient per parameter]
so the partition and reduction logic is exercised with gloo ranks on the CPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["probe_range", "slq_logdet_sharded", "sharded_slq", "Communicator", "partition_rows",
           "PartitionedEigsh"]


def probe_range(p_total: int, rank: int, world: int):
    """Contiguous balanced share [c0, c1) of p_total probe columns for `rank`."""
    base, extra = divmod(p_total, world)
    c0 = rank * base + min(rank, extra)
    return c0, c0 + base + (1 if rank < extra else 0)


class _ShardedSLQ(torch.autograd.Function):
    @staticmethod
    def forward(ctx, engine, Z_local, p_total: int, group, *params):
        need = any(ctx.needs_input_grad[4:])
        if Z_local.shape[1] > 0:
            total, state = engine.forward(Z_local, p_total, keep=need)
        else:
            total, state = torch.zeros((), dtype=torch.float64), []
        t = total.detach().to(torch.float64).reshape(1).clone()
        t = t.to(_comm_device(group, None))
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        ctx.engine, ctx.state, ctx.group, ctx.empty = engine, state, group, Z_local.shape[1] == 0
        ctx.pinfo = [(p.device, p.dtype, p.shape) for p in params]
        ref = params[0] if params else t
        return (t[0] / p_total).to(ref.device, ref.dtype)

    @staticmethod
    def backward(ctx, g):
        n_par = len(ctx.pinfo)
        if ctx.empty:
            local = [torch.zeros((), dtype=torch.float64) for _ in range(n_par)]
        else:
            dev = _engine_device(ctx.engine)
            g_out = g.detach().to(dev, torch.float64).reshape(1)
            local = ctx.engine.backward(ctx.state, g_out)
        cdev = _comm_device(ctx.group, None)
        flat = torch.stack([torch.as_tensor(x).to(cdev, torch.float64).reshape(()) if x is not None
                            else torch.zeros((), dtype=torch.float64, device=cdev) for x in local])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=ctx.group)
        ctx.state = None
        out = [flat[k].to(d, dt).reshape(sh) for k, (d, dt, sh) in enumerate(ctx.pinfo)]
        return (None, None, None, None, *out)


def _comm_device(group, _):
    backend = dist.get_backend(group)
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _engine_device(engine):
    mv = getattr(engine, "mv", None)
    return getattr(mv, "device", torch.device("cpu"))


def sharded_slq(engine, Z_full, params, group=None):
    """Run `engine` on this rank's share of the probe columns of Z_full and
    combine across the group (see module docstring)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    p_total = Z_full.shape[1]
    c0, c1 = probe_range(p_total, rank, world)
    return _ShardedSLQ.apply(engine, Z_full[:, c0:c1], p_total, group, *params)


def slq_logdet_sharded(matvec, n, params, m_probes=20, lanczos_m=50, seed=0, dtype=torch.float64, group=None):
    """slq_logdet of an IMGP precision operator with the probes split over the
    ranks of `group` (default: the world).  Every rank gets the full estimate
    and the full parameter gradients."""
    from .funm_torch import _probes
    from .imgp import ImgpPrecisionMatvec, ImgpSLQEngine, _scalar

    if not isinstance(matvec, ImgpPrecisionMatvec) or len(params) != 2:
        raise TypeError("slq_logdet_sharded runs the fused engine: matvec must come from "
                        "make_imgp_precision_matvec and params must be (lengthscale, graphbandwidth)")
    params = tuple(params)
    Z = _probes(n, m_probes, seed, dtype, matvec.device).to(matvec.dtype)
    engine = ImgpSLQEngine(matvec, lanczos_m, _scalar(params[0]), _scalar(params[1]))
    return sharded_slq(engine, Z, params, group)


# ---------------------------------------------------------------------------
# Row-partitioned eigsh
# ---------------------------------------------------------------------------
def partition_rows(n: int, world: int, rank: int):
    """Global rows [r0, r1) owned by `rank` (block size from the engine)."""
    from . import _native

    nb = _native.lib.lg_partition_block(int(n), int(world))
    r0 = min(rank * nb, n)
    return r0, min(r0 + nb, n)


class Communicator:
    """The engine's NCCL communicator over the ranks of a torch.distributed
    group: rank 0 draws the unique id, the group broadcasts it."""

    def __init__(self, group=None):
        import ctypes as C

        from . import _native

        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        obj = [None]
        if self.rank == 0:
            buf = C.create_string_buffer(128)
            _native.check(_native.lib.lg_comm_unique_id(buf, 128))
            obj = [bytes(buf.raw)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        h = C.c_void_p()
        _native.check(_native.lib.lg_comm_create(C.byref(h), obj[0], 128, self.world, self.rank))
        self.handle = h

    def close(self):
        from . import _native

        if self.handle is not None and self.handle.value:
            _native.lib.lg_comm_destroy(self.handle)
        self.handle = None


class PartitionedEigsh:
    """eigsh of an n x n matrix whose rows are split over the ranks.

    rowptr, col, vals: this rank's rows [r0, r1) (see partition_rows) as a CSR
    with global column indices, torch tensors on this rank's GPU (int32,
    int32, float64).  solve() takes the keywords of gpu_eigsh.EigshPlan.solve
    with v0 = this rank's slice and returns (eigenvalues, this rank's rows of
    the eigenvectors as an (r1 - r0) x k tensor)."""

    def __init__(self, comm: Communicator, n_global: int, rowptr, col, vals, max_ncv: int = 127,
                 mixed: bool = False, exchange: str = "auto", transport: str = "auto"):
        import torch

        from . import EigshPlan

        self.comm, self.n_global = comm, int(n_global)
        self.r0, self.r1 = partition_rows(n_global, comm.world, comm.rank)
        n_local = self.r1 - self.r0
        if rowptr.numel() != n_local + 1:
            raise ValueError(f"rank {comm.rank} must pass rows [{self.r0}, {self.r1}) ({n_local} rows)")
        self._keep = (rowptr, col, vals)
        self.plan = EigshPlan(None, max_ncv=max_ncv, mixed=mixed, comm=comm, n_global=n_global,
                              device_csr=(n_local, int(col.numel()), rowptr.data_ptr(), col.data_ptr(),
                                          vals.data_ptr()))
        self.device = vals.device
        self.torch = torch
        if exchange != "auto":
            self.set_exchange(exchange)
        if transport != "auto":
            self.set_transport(transport)

    def set_transport(self, mode: str):
        """'auto', 'nccl' or 'peer' (every rank must choose the same): how the
        partial sums are reduced and the residual rows exchanged — NCCL
        collectives, or one kernel each that stores into the other ranks'
        memory over NVLink."""
        from . import _native

        if mode not in _native.TRANSPORT:
            raise ValueError("transport must be 'auto', 'nccl' or 'peer'")
        _native.check(_native.lib.lg_eigsh_plan_set_transport(self.plan._plan, _native.TRANSPORT[mode]))

    @property
    def transport(self) -> str:
        import ctypes as C

        from . import _native

        m = C.c_int(0)
        _native.check(_native.lib.lg_eigsh_plan_transport(self.plan._plan, C.byref(m)))
        return {v: k for k, v in _native.TRANSPORT.items()}[m.value]

    def set_exchange(self, mode: str):
        """'auto', 'allgather' or 'halo' (every rank must choose the same)."""
        from . import _native

        if mode not in _native.EXCHANGE:
            raise ValueError("exchange must be 'auto', 'allgather' or 'halo'")
        _native.check(_native.lib.lg_eigsh_plan_set_exchange(self.plan._plan, _native.EXCHANGE[mode]))

    @property
    def exchange_info(self):
        """(mode, rows received from other ranks, rows sent to them) per sparse product."""
        import ctypes as C

        from . import _native

        m, r, s = C.c_int(0), C.c_longlong(0), C.c_longlong(0)
        _native.check(_native.lib.lg_eigsh_plan_exchange_info(self.plan._plan, C.byref(m), C.byref(r), C.byref(s)))
        names = {v: k for k, v in _native.EXCHANGE.items()}
        return names[m.value], int(r.value), int(s.value)

    def solve(self, k, v0_local, **kw):
        torch = self.torch
        v0 = torch.as_tensor(v0_local, dtype=torch.float64).to(self.device).contiguous()
        Y = torch.empty((self.r1 - self.r0, int(k)), dtype=torch.float64, device=self.device)
        w, _ = self.plan.solve(k=k, v0_device=v0.data_ptr(), evecs_out=Y.data_ptr(), **kw)
        return w, Y

    @property
    def last_info(self):
        return self.plan.last_info

    def close(self):
        self.plan.close()
