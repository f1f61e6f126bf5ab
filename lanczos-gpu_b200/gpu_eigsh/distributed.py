"""Multi-GPU stochastic Lanczos quadrature: probes sharded across ranks.

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

__all__ = ["probe_range", "slq_logdet_sharded", "sharded_slq"]


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
