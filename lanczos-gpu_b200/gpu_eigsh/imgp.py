"""IMGP graph-Matern precision operator on the GPU.

``make_imgp_precision_matvec(*, x_edge_dists, idx, operator_dim, nu,
normalization="symmetric", self_loops=True)`` returns a callable
``matvec(rhs, lengthscale, graphbandwidth)`` computing

    P(theta, kappa) rhs = (2 nu / theta^2 I + L_sym(kappa))^nu rhs

for rhs of shape (n,) or (n, B), differentiable with respect to rhs,
lengthscale (theta) and graphbandwidth (kappa) — the interface of the
reference's make_imgp_precision_matvec (python/gpu_eigsh/imgp.py:234-289).

How it runs:
  * the edge list (idx (2, M), one entry per undirected edge) becomes, once,
    a device CSR that stores every edge in both directions, with the squared
    edge distances permuted into CSR order;
  * L_sym(kappa) and dL/dkappa are built by the CUDA kernels of
    lg_imgp_laplacian (the reference's _build_laplacian_cache, imgp.py:142-189)
    and cached for the last kappa value;
  * P X runs as nu fused sparse products (lg_slq_apply), its VJP as
    lg_slq_apply_vjp; gradients reach kappa through dL/dkappa and theta
    through d(2 nu / theta^2)/dtheta;
  * slq_logdet (gpu_eigsh.funm_torch) recognises this object and runs the whole
    stochastic Lanczos quadrature and its Kraemer backward on the fused kernels
    (``_slq_logdet_fused``).

Inputs may live on the CPU (as in the reference's examples); the operator is
moved to the current CUDA device and results come back on the device of rhs.
There is no CPU implementation: without CUDA the constructor raises.
"""
from __future__ import annotations

import math

import torch

from . import _native, _slq

__all__ = ["make_imgp_precision_matvec", "ImgpPrecisionMatvec", "_matmul_symmetric_laplacian",
           "imgp_neg_marginal_log_likelihood"]

_MAXB = 128


def _scalar(t) -> float:
    return float(t.detach().reshape(-1)[0]) if torch.is_tensor(t) else float(t)


class ImgpPrecisionMatvec:
    """Callable P(theta, kappa) X on the GPU; see the module docstring."""

    def __init__(self, x_edge_dists, idx, operator_dim: int, nu: int, self_loops: bool = True,
                 reorder: bool = True):
        dev = _slq.require_cuda()
        d2 = torch.as_tensor(x_edge_dists).detach()
        if d2.is_cuda:
            dev = d2.device
        d2 = d2.to(dev)
        if d2.dtype not in (torch.float32, torch.float64):
            d2 = d2.to(torch.float64)
        idx = torch.as_tensor(idx).to(dev, torch.int64)
        if idx.dim() != 2 or idx.shape[0] != 2 or idx.shape[1] != d2.numel():
            raise ValueError("idx must be (2, M) with one squared distance per edge")
        n = int(operator_dim)
        if nu < 1 or nu > 8 or int(nu) != nu:
            raise ValueError("nu must be an integer in [1, 8]")
        M = idx.shape[1]
        if 2 * M >= 2 ** 31 or n >= 2 ** 31:
            raise ValueError("graph too large for int32 CSR indices")
        if M and (int(idx.min()) < 0 or int(idx.max()) >= n):
            raise ValueError("edge index out of range [0, operator_dim)")
        self.n, self.nu, self.self_loops = n, int(nu), bool(self_loops)
        self.dtype = d2.dtype
        self.device = dev
        rows = torch.cat([idx[0], idx[1]])
        cols = torch.cat([idx[1], idx[0]])
        eid = torch.arange(M, device=dev).repeat(2)
        self.rowptr, self.col, self.d2 = self._csr(rows, cols, eid, d2)
        # row order for locality of the neighbour gathers: Cuthill-McKee from
        # a peripheral vertex; perm[new] = old, pos[old] = new
        self.perm = self.pos = None
        if reorder and M:
            perm = self._bfs_order()
            pos = torch.empty_like(perm)
            pos[perm] = torch.arange(n, device=dev)
            self.rowptr, self.col, self.d2 = self._csr(pos[rows], pos[cols], eid, d2)
            self.perm, self.pos = perm, pos
        self.nnz = int(self.col.numel())
        self._lap_key = None
        self._lap = None

    def _csr(self, rows, cols, eid, d2):
        """CSR (rows sorted by (row, col)) with the squared distance of every entry."""
        n = self.n
        order = torch.argsort(rows * n + cols, stable=True)
        counts = torch.bincount(rows, minlength=n)
        rowptr = torch.zeros(n + 1, dtype=torch.int32, device=self.device)
        rowptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
        return rowptr, cols[order].to(torch.int32).contiguous(), d2[eid[order]].contiguous()

    def _bfs_order(self) -> torch.Tensor:
        """Cuthill-McKee order of the graph (gpu_eigsh.ordering.cm_order):
        BFS levels from a pseudo-peripheral vertex, each level in the order of
        the vertices that found it (8-9 % faster SLQ products at n = 1e6 than
        the levels alone)."""
        from .ordering import cm_order

        return cm_order(self.rowptr, self.col)

    def to_internal(self, X: torch.Tensor) -> torch.Tensor:
        """Rows of X (caller's vertex order) in the operator's row order."""
        return X if self.perm is None else X.index_select(0, self.perm)

    def to_caller(self, Y: torch.Tensor) -> torch.Tensor:
        return Y if self.pos is None else Y.index_select(0, self.pos)

    # -- L_sym(kappa) and dL/dkappa -----------------------------------------------
    def laplacian(self, kappa: float):
        """(offval (nnz,), diag (n,), doffval, ddiag) for graphbandwidth kappa, cached."""
        if self._lap_key != kappa:
            off = torch.empty(self.nnz, dtype=self.dtype, device=self.device)
            doff = torch.empty_like(off)
            diag = torch.empty(self.n, dtype=self.dtype, device=self.device)
            ddiag = torch.empty_like(diag)
            work = torch.empty(4 * self.n, dtype=torch.float64, device=self.device)
            _native.check(_native.lib.lg_imgp_laplacian(
                self.n, self.nnz, self.rowptr.data_ptr(), self.col.data_ptr() if self.nnz else None,
                _slq.dtype_code(self.dtype), self.d2.data_ptr() if self.nnz else None, float(kappa),
                int(self.self_loops), off.data_ptr() if self.nnz else None, diag.data_ptr(),
                doff.data_ptr() if self.nnz else None, ddiag.data_ptr(), work.data_ptr(),
                _slq.stream(self.device)))
            self._lap_key, self._lap = kappa, (off, diag, doff, ddiag)
        return self._lap

    def operator(self, lengthscale: float, kappa: float) -> _slq.Operator:
        off, diag, doff, ddiag = self.laplacian(kappa)
        shift = 2.0 * self.nu / (lengthscale * lengthscale)
        return _slq.Operator(self.n, self.rowptr, self.col, off, diag, doff, ddiag, shift, self.nu, self.dtype)

    def shift_derivative(self, lengthscale: float) -> float:
        """d(2 nu / theta^2) / d theta."""
        return -4.0 * self.nu / lengthscale ** 3

    def __call__(self, rhs, lengthscale, graphbandwidth):
        return _PrecisionApply.apply(rhs, lengthscale, graphbandwidth, self)


def _column_chunks(B: int):
    k = (B + _MAXB - 1) // _MAXB
    step = (B + k - 1) // k
    return [(c, min(B, c + step)) for c in range(0, B, step)]


def _blocked(X: torch.Tensor, dev, dtype):
    """(n, B) -> list of (block (n, ld), b) per chunk of <= 128 columns."""
    out = []
    for c0, c1 in _column_chunks(X.shape[1]):
        blk, b, _ = _slq.to_block(X[:, c0:c1], dev, dtype)
        out.append((blk, b))
    return out


class _PrecisionApply(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rhs, lengthscale, graphbandwidth, mv: ImgpPrecisionMatvec):
        ell, kap = _scalar(lengthscale), _scalar(graphbandwidth)
        op = mv.operator(ell, kap)
        X2 = rhs.reshape(-1, 1) if rhs.dim() == 1 else rhs
        if X2.shape[0] != mv.n:
            raise ValueError(f"rhs has {X2.shape[0]} rows, the operator {mv.n}")
        parts = _blocked(mv.to_internal(X2.detach().to(mv.device, mv.dtype)), mv.device, mv.dtype)
        outs = [op.apply(blk, b, blk.shape[1])[:, :b] for blk, b in parts]
        Y = mv.to_caller(torch.cat(outs, dim=1) if len(outs) > 1 else outs[0])
        ctx.mv, ctx.ell, ctx.kap, ctx.shape = mv, ell, kap, rhs.shape
        ctx.rhs_dev, ctx.rhs_dtype = rhs.device, rhs.dtype
        ctx.parts = parts
        ctx.pdev = (lengthscale.device if torch.is_tensor(lengthscale) else None,
                    graphbandwidth.device if torch.is_tensor(graphbandwidth) else None)
        ctx.pshape = (lengthscale.shape if torch.is_tensor(lengthscale) else None,
                      graphbandwidth.shape if torch.is_tensor(graphbandwidth) else None)
        ctx.pdtype = (lengthscale.dtype if torch.is_tensor(lengthscale) else None,
                      graphbandwidth.dtype if torch.is_tensor(graphbandwidth) else None)
        return Y.reshape(rhs.shape).to(rhs.device, rhs.dtype)

    @staticmethod
    def backward(ctx, g):
        mv = ctx.mv
        op = mv.operator(ctx.ell, ctx.kap)
        G2 = g.reshape(-1, 1) if g.dim() == 1 else g
        gparts = _blocked(mv.to_internal(G2.detach().to(mv.device, mv.dtype)), mv.device, mv.dtype)
        gxs, gp = [], torch.zeros(2, dtype=torch.float64, device=mv.device)
        for (blk, b), (gblk, _) in zip(ctx.parts, gparts):
            gX, gpp = op.apply_vjp(blk, gblk, b, blk.shape[1])
            gxs.append(gX[:, :b])
            gp = gp + gpp
        g_rhs = mv.to_caller(torch.cat(gxs, dim=1) if len(gxs) > 1 else gxs[0])
        g_rhs = g_rhs.reshape(ctx.shape).to(ctx.rhs_dev, ctx.rhs_dtype)
        g_ell = gp[1] * mv.shift_derivative(ctx.ell)
        g_kap = gp[0]
        out = [g_rhs]
        for k, gv in enumerate((g_ell, g_kap)):
            if ctx.pdev[k] is None:
                out.append(None)
            else:
                out.append(gv.to(ctx.pdev[k], ctx.pdtype[k]).reshape(ctx.pshape[k]))
        return out[0], out[1], out[2], None


def make_imgp_precision_matvec(*, x_edge_dists, idx, operator_dim, nu, normalization="symmetric",
                               self_loops=True):
    """P(kappa, theta) = (2 nu / theta^2 I + L_sym(kappa))^nu as a differentiable
    callable ``matvec(rhs, lengthscale, graphbandwidth)`` (imgp.py:234-289)."""
    if normalization != "symmetric":
        raise NotImplementedError(
            "Only normalization='symmetric' is implemented (the case used by SS-IMGP-full).")
    return ImgpPrecisionMatvec(x_edge_dists, idx, operator_dim, nu, self_loops)


def _matmul_symmetric_laplacian(rhs, x_edge_dists, idx, operator_dim, graphbandwidth, self_loops=True):
    """L_sym(kappa) rhs (the reference's one-shot helper, imgp.py:210-226): the
    power-1 operator with zero shift."""
    mv = ImgpPrecisionMatvec(x_edge_dists, idx, operator_dim, 1, self_loops, reorder=False)
    kap = _scalar(graphbandwidth)
    off, diag, doff, ddiag = mv.laplacian(kap)
    op = _slq.Operator(mv.n, mv.rowptr, mv.col, off, diag, doff, ddiag, 0.0, 1, mv.dtype)
    X2 = rhs.reshape(-1, 1) if rhs.dim() == 1 else rhs
    outs = [op.apply(blk, b, blk.shape[1])[:, :b] for blk, b in _blocked(X2.detach(), mv.device, mv.dtype)]
    Y = torch.cat(outs, dim=1) if len(outs) > 1 else outs[0]
    return Y.reshape(rhs.shape).to(rhs.device, rhs.dtype)


# ---------------------------------------------------------------------------
# Fused stochastic Lanczos quadrature on this operator
# ---------------------------------------------------------------------------
class ImgpSLQEngine:
    """The fused SLQ of one probe set on one GPU, split into a forward that
    returns the sum of the per-probe quadratures and a backward that returns
    the gradient of that sum with respect to (lengthscale, graphbandwidth).
    `p_total` is the number of probes of the whole estimate (the mean divides by
    it), so that shards of the probes on several GPUs add up."""

    def __init__(self, mv: ImgpPrecisionMatvec, lanczos_m: int, lengthscale: float, graphbandwidth: float):
        self.mv, self.m = mv, int(lanczos_m)
        self.ell, self.kap = float(lengthscale), float(graphbandwidth)

    def forward(self, Z, p_total: int, keep: bool = True):
        """Z: (n, b) probes in the caller's vertex order.  Returns (sum_b q_b as
        a 0-d fp64 tensor, state for backward)."""
        mv = self.mv
        op = mv.operator(self.ell, self.kap)
        q_all, saved = [], []
        for blk, b in _blocked(mv.to_internal(Z), mv.device, mv.dtype):
            ld = blk.shape[1]
            V, Y, alpha, beta, znorm = op.forward(blk, b, ld, self.m)
            q, ga, gb, _ = _slq.small_side(alpha, beta, znorm, "log", 0, g_scale=1.0 / p_total)
            q_all.append(q)
            if keep:
                saved.append((V, Y, alpha, beta, ga, gb, b, ld))
        return torch.cat(q_all).sum(), saved

    def backward(self, saved, g_out):
        """g_out: gradient of the loss with respect to the mean (fp64, 1 element
        on the operator's device).  Returns [d/d lengthscale, d/d graphbandwidth]
        of this shard's contribution as fp64 device tensors."""
        mv = self.mv
        op = mv.operator(self.ell, self.kap)
        gp = torch.zeros(2, dtype=torch.float64, device=mv.device)
        for V, Y, alpha, beta, ga, gb, b, ld in saved:
            gp = gp + op.backward(V, Y, alpha, beta, ga, gb, g_out, b, ld, self.m)
        return [gp[1] * mv.shift_derivative(self.ell), gp[0]]


def _param_info(params):
    return [(t.device, t.dtype, t.shape) if torch.is_tensor(t) else None for t in params]


def _grads_to_params(grads, pinfo):
    return [None if info is None else g.to(info[0], info[1]).reshape(info[2]) for g, info in zip(grads, pinfo)]


class _SLQImgp(torch.autograd.Function):
    """log det P(theta, kappa) by SLQ over the probe columns of Z, with the
    Kraemer backward, entirely on the fused kernels (lg_slq_forward /
    lg_slq_small_side / lg_slq_backward).  Follows _SLQLogdetBatched
    (python/gpu_eigsh/funm_torch.py:571-727)."""

    @staticmethod
    def forward(ctx, mv: ImgpPrecisionMatvec, Z, lanczos_m: int, lengthscale, graphbandwidth):
        eng = ImgpSLQEngine(mv, lanczos_m, _scalar(lengthscale), _scalar(graphbandwidth))
        need = any(ctx.needs_input_grad[3:5])
        total, saved = eng.forward(Z, Z.shape[1], keep=need)
        ctx.eng, ctx.saved = eng, saved
        ctx.pinfo = _param_info((lengthscale, graphbandwidth))
        return (total / Z.shape[1]).to(Z.dtype)

    @staticmethod
    def backward(ctx, g_ld):
        eng = ctx.eng
        g_out = g_ld.detach().to(eng.mv.device, torch.float64).reshape(1)
        grads = eng.backward(ctx.saved, g_out)
        ctx.saved = None
        out = _grads_to_params(grads, ctx.pinfo)
        return None, None, None, out[0], out[1]


def _slq_logdet_fused(mv: ImgpPrecisionMatvec, Z, lanczos_m, lengthscale, graphbandwidth):
    return _SLQImgp.apply(mv, Z, lanczos_m, lengthscale, graphbandwidth)


# ---------------------------------------------------------------------------
# Marginal likelihood
# ---------------------------------------------------------------------------
_OPERATOR_CACHE: dict = {}


def _cached_operator(x_edge_dists, idx, n, nu, self_loops):
    """The operator of (x_edge_dists, idx, n, nu, self_loops), built once: the
    CSR assembly and the Cuthill-McKee renumbering cost more than a log-det, and
    a training loop calls with the same graph every iteration.  Keyed by the
    tensors' storage, shape and version counter (an in-place change rebuilds);
    one entry is kept."""
    def key_of(t):
        t = torch.as_tensor(t)
        return (t.device, t.dtype, tuple(t.shape), t.data_ptr(), t._version)

    key = (key_of(x_edge_dists), key_of(idx), int(n), int(nu), bool(self_loops))
    mv = _OPERATOR_CACHE.get(key)
    if mv is None:
        _OPERATOR_CACHE.clear()
        mv = ImgpPrecisionMatvec(x_edge_dists, idx, n, nu, self_loops)
        _OPERATOR_CACHE[key] = mv
    return mv


def imgp_neg_marginal_log_likelihood(train_targets: torch.Tensor, *, x_edge_dists: torch.Tensor, idx: torch.Tensor,
                                     operator_dim: int, nu: int, lengthscale: torch.Tensor,
                                     graphbandwidth: torch.Tensor, m_probes: int = 20, lanczos_m: int = 50,
                                     seed: int = 0, normalization: str = "symmetric",
                                     self_loops: bool = True) -> torch.Tensor:
    """Per-data-point negative log marginal likelihood of the precision-
    parameterised graph GP (the reference's imgp.py:296-341):

        (1 / N) * 0.5 * (y^T P y - log det P + N log 2 pi),

    y^T P y exact through the fused precision product, log det P by the fused
    SLQ (m_probes Rademacher probes, Lanczos depth lanczos_m), both
    differentiable in lengthscale and graphbandwidth.  The operator is built
    once per graph and reused across calls.
    """
    if normalization != "symmetric":
        raise NotImplementedError(
            "Only normalization='symmetric' is implemented (the case used by SS-IMGP-full).")
    from .funm_torch import slq_logdet

    n = int(operator_dim)
    matvec = _cached_operator(x_edge_dists, idx, n, nu, self_loops)
    Py = matvec(train_targets, lengthscale, graphbandwidth)
    inv_quad = torch.dot(train_targets.reshape(-1), Py.reshape(-1).to(train_targets.dtype))
    logdet = slq_logdet(matvec, n, (lengthscale, graphbandwidth), m_probes=m_probes, lanczos_m=lanczos_m, seed=seed,
                        dtype=train_targets.dtype, device=train_targets.device)
    log_2pi = math.log(2.0 * math.pi)
    nll = 0.5 * (inv_quad - logdet.to(inv_quad.dtype) + n * log_2pi)
    return nll / n

