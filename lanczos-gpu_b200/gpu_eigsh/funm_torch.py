"""Differentiable matrix functions by Lanczos quadrature, on the GPU.

Same names, arguments and results as the reference module
python/gpu_eigsh/funm_torch.py:

  slq_logdet(matvec, n, params, m_probes=20, lanczos_m=50, seed=0,
             dtype=torch.float64, device="cpu", batched=True)      (:730-781)
  funm_apply_kraemer(A, v, m, func="log")                           (:254-373)
  funm_qform_op(matvec, z, params, m, func="log")                   (:380-564)
  lanczos_torch_noreortho(matvec, v, m)                              (:83-117)
  lanczos_torch_noreortho_batched(matvec_batched, Z, m)              (:120-173)
  _small_side, _build_T, _apply_scalar                               (:41-76)

Execution:
  * The three-term recurrence, its column dots and norms, the per-probe
    small side (tridiagonal eigen-decomposition, quadrature and its
    Daleckii-Krein gradient) and every Kraemer reverse step run in the CUDA
    library (lg_slq_block_*, lg_slq_small_side).  Only the caller's own
    matvec (and, in the backward, autograd through it for the parameter
    gradient, as in the reference) runs outside it, on the device where the
    caller's tensors live.
  * slq_logdet with an operator from gpu_eigsh.imgp.make_imgp_precision_matvec
    runs entirely on the fused sparse kernels (no Python per step).
  * funm_apply_kraemer multiplies by the dense A with the library's dense
    matvec and accumulates grad_A = sum_j lambda_j x_j^T on the GPU.

Probes of slq_logdet are drawn exactly as the reference draws them (torch CPU
generator, randint(0, 2) * 2 - 1) and kept on the GPU for repeated calls with
the same (n, m_probes, seed, dtype).  There is no CPU implementation: every
entry point needs a CUDA device.
"""
from __future__ import annotations

import torch

from . import _slq

__all__ = ["slq_logdet", "funm_apply_kraemer", "funm_qform_op", "lanczos_torch_noreortho",
           "lanczos_torch_noreortho_batched", "_small_side", "_build_T", "_apply_scalar"]


# ---------------------------------------------------------------------------
# Small helpers with the reference's semantics
# ---------------------------------------------------------------------------
def _apply_scalar(theta: torch.Tensor, func: str) -> torch.Tensor:
    if func == "log":
        return torch.log(theta)
    if func == "exp":
        return torch.exp(theta)
    if func == "sqrt":
        return torch.sqrt(theta)
    if func == "inv":
        return 1.0 / theta
    raise ValueError(f"unknown func: {func}")


def _build_T(alpha: torch.Tensor, beta_sub: torch.Tensor) -> torch.Tensor:
    """Symmetric tridiagonal m x m from its diagonal and subdiagonal."""
    m = alpha.shape[0]
    T = torch.diag(alpha)
    if m > 1:
        T = T + torch.diag(beta_sub, diagonal=1) + torch.diag(beta_sub, diagonal=-1)
    return T


def _check_func(func: str):
    if func not in ("log", "exp", "sqrt", "inv"):
        raise ValueError(f"unknown func: {func}")


def _small_side(V: torch.Tensor, alpha: torch.Tensor, beta_sub: torch.Tensor, v_norm, func: str):
    """y = v_norm * V f(T) e1 with T = tridiag(alpha, beta_sub) (not differentiable;
    the autograd Functions below carry the gradients)."""
    _check_func(func)
    dev = _slq.require_cuda()
    m = alpha.shape[0]
    a = alpha.detach().to(dev, torch.float64).reshape(1, m).contiguous()
    b = torch.zeros((1, m), dtype=torch.float64, device=dev)
    if m > 1:
        b[0, :m - 1] = beta_sub.detach().to(dev, torch.float64)
    u, _, _, _ = _slq.small_side(a, b, None, func, 1)
    u = u[0].to(V.device, V.dtype)
    return v_norm * (V @ u)


# ---------------------------------------------------------------------------
# Recurrence around a caller-supplied product
# ---------------------------------------------------------------------------
class _Basis:
    """Device blocks (k, n, ld) of the recurrence plus the caller's matvec I/O."""

    def __init__(self, n: int, B: int, m: int, dtype, user_device):
        self.dev = _slq.require_cuda()
        self.n, self.B, self.m, self.dtype = n, B, m, dtype
        self.ld = _slq.ld_for(B, dtype)
        self.user_device = torch.device(user_device)
        self.rec = _slq.BlockRecurrence(n, B, self.ld, dtype, self.dev)
        self.V = _slq.blocks(m + 1, n, self.ld, dtype, self.dev)
        self.R = _slq.blocks(1, n, self.ld, dtype, self.dev)[0]
        self.W = _slq.blocks(1, n, self.ld, dtype, self.dev, zero=True)[0]
        self.alpha = torch.empty((B, m), dtype=torch.float64, device=self.dev)
        self.beta = torch.empty((B, m), dtype=torch.float64, device=self.dev)
        self.znorm = torch.empty(B, dtype=torch.float64, device=self.dev)

    def user(self, blk: torch.Tensor, vector: bool):
        x = blk[:, 0] if vector else blk[:, :self.B]
        return x.to(self.user_device)

    def load(self, dst: torch.Tensor, y: torch.Tensor):
        y2 = y.reshape(self.n, -1) if y.dim() == 1 else y
        if y2.shape != (self.n, self.B):
            raise ValueError(f"matvec returned shape {tuple(y.shape)}, expected ({self.n}, {self.B})")
        dst[:, :self.B].copy_(y2)
        return dst

    def run(self, Z: torch.Tensor, mv, vector: bool):
        """m steps from the probe block Z (on the device); mv(x_user) -> P x_user."""
        self.rec.start(Z, self.V[0], self.znorm)
        for j in range(self.m):
            W = self.load(self.W, mv(self.user(self.V[j], vector)))
            self.rec.step(j, self.m, W, self.V[j], self.V[j - 1] if j > 0 else None, self.R, self.V[j + 1],
                          self.alpha, self.beta)


def lanczos_torch_noreortho(matvec, v: torch.Tensor, m: int):
    """Three-term Lanczos without reorthogonalisation of one vector:
    (V_full (n, m+1), alpha (m,), betas (m,), v_norm)."""
    n = v.shape[0]
    bs = _Basis(n, 1, m, v.dtype, v.device)
    Z, _, _ = _slq.to_block(v.detach(), bs.dev, v.dtype)
    bs.run(Z, matvec, vector=True)
    V = bs.V[:, :, 0].T.to(v.device)
    return V, bs.alpha[0].to(v.device, v.dtype), bs.beta[0].to(v.device, v.dtype), bs.znorm[0].to(v.device, v.dtype)


def lanczos_torch_noreortho_batched(matvec_batched, Z: torch.Tensor, m: int):
    """B independent three-term Lanczos runs: (V_full (n, B, m+1), alpha (B, m),
    betas (B, m), Z_norm (B,))."""
    n, B = Z.shape
    if B > 128:
        raise ValueError("lanczos_torch_noreortho_batched: at most 128 columns per call")
    bs = _Basis(n, B, m, Z.dtype, Z.device)
    Zb, _, _ = _slq.to_block(Z.detach(), bs.dev, Z.dtype)
    bs.run(Zb, matvec_batched, vector=False)
    V = bs.V[:, :, :B].permute(1, 2, 0).contiguous().to(Z.device)
    return (V, bs.alpha.to(Z.device, Z.dtype), bs.beta.to(Z.device, Z.dtype), bs.znorm.to(Z.device, Z.dtype))


def _param_vjp(matvec, x_user, params, lam_user):
    """d<lam, matvec(x, *params)>/d params by autograd through the caller's matvec
    (funm_torch.py:690-703)."""
    if not params:
        return []
    pd = tuple(p.detach().clone().requires_grad_(True) for p in params)
    with torch.enable_grad():
        out = matvec(x_user.detach(), *pd)
        return list(torch.autograd.grad(out, pd, grad_outputs=lam_user.detach().reshape(out.shape),
                                        allow_unused=True))


def _reverse_sweep(bs: _Basis, matvec, params, g_alpha, g_beta, g_out, vector: bool, need_xi0: bool,
                   dcoef=None, G=None, on_lambda=None, plam=None):
    """Kraemer reverse sweep over the stored basis.  Returns (param grads, xi of
    the final step or None).  matvec(x_user, *params) is the caller's operator;
    plam(lam_block, out_block) may replace it for P lambda."""
    m, dev = bs.m, bs.dev
    grads = [None] * len(params)
    xi = _slq.blocks(1, bs.n, bs.ld, bs.dtype, dev)[0]
    lam = _slq.blocks(1, bs.n, bs.ld, bs.dtype, dev)[0]
    lplus = _slq.blocks(1, bs.n, bs.ld, bs.dtype, dev)[0]
    Pl = bs.W
    for j in range(m - 1, -1, -1):
        bs.rec.lam(j, m, xi if j < m - 1 else None, bs.V[j + 1], bs.V[j], bs.beta, g_alpha, g_beta, g_out, lam)
        if on_lambda is not None:
            on_lambda(lam, bs.V[j])
        if params:
            gp = _param_vjp(lambda x, *p: matvec(x, *p), bs.user(bs.V[j], vector), params, bs.user(lam, vector))
            for k, g in enumerate(gp):
                if g is not None:
                    grads[k] = g if grads[k] is None else grads[k] + g
        if j > 0 or need_xi0:
            if plam is not None:
                plam(lam, Pl)
            else:
                with torch.no_grad():
                    bs.load(Pl, matvec(bs.user(lam, vector), *params))
            dc = None if dcoef is None else dcoef[:, j].contiguous()
            bs.rec.xi(j, m, Pl, lam, lplus if j < m - 1 else None, bs.V[j + 1], bs.V[j],
                      bs.V[j - 1] if j > 0 else None, bs.alpha, bs.beta, dc, G, xi)
        lam, lplus = lplus, lam
    return grads, (xi if need_xi0 else None)


def _grads_like(grads, params):
    out = []
    for g, p in zip(grads, params):
        if g is None:
            out.append(None)
        else:
            out.append(g.to(p.device, p.dtype).reshape(p.shape) if torch.is_tensor(p) else g)
    return out


# ---------------------------------------------------------------------------
# Stochastic Lanczos quadrature (generic operator)
# ---------------------------------------------------------------------------
class _SLQLogdetBatched(torch.autograd.Function):
    """log det by SLQ over the columns of Z with a caller-supplied batched matvec
    (funm_torch.py:571-727); recurrence, small side and reverse sweep in CUDA."""

    @staticmethod
    def forward(ctx, matvec, Z, lanczos_m, *params):
        n, P = Z.shape
        m = int(lanczos_m)
        chunks = []
        q_all = []
        for c0, c1 in _chunk_ranges(P):
            bs = _Basis(n, c1 - c0, m, Z.dtype, Z.device)
            Zb, _, _ = _slq.to_block(Z[:, c0:c1].detach(), bs.dev, Z.dtype)
            with torch.no_grad():
                bs.run(Zb, lambda X: matvec(X, *params), vector=False)
            q, ga, gb, _ = _slq.small_side(bs.alpha, bs.beta, bs.znorm, "log", 0, g_scale=1.0 / P)
            q_all.append(q)
            chunks.append((bs, ga, gb))
        ctx.chunks, ctx.matvec = chunks, matvec
        ctx.save_for_backward(*params)
        return (torch.cat(q_all).sum() / P).to(Z.device, Z.dtype)

    @staticmethod
    def backward(ctx, g_ld):
        params = ctx.saved_tensors
        grads = [None] * len(params)
        for bs, ga, gb in ctx.chunks:
            g_out = g_ld.detach().to(bs.dev, torch.float64).reshape(1)
            gp, _ = _reverse_sweep(bs, ctx.matvec, params, ga, gb, g_out, vector=False, need_xi0=False)
            for k, g in enumerate(gp):
                if g is not None:
                    grads[k] = g if grads[k] is None else grads[k] + g
        ctx.chunks = None
        return (None, None, None, *_grads_like(grads, params))


def _chunk_ranges(P: int):
    k = (P + 127) // 128
    step = (P + k - 1) // k
    return [(c, min(P, c + step)) for c in range(0, P, step)]


_PROBES: dict = {}


def _probes(n: int, m_probes: int, seed: int, dtype, device):
    """Rademacher probes exactly as funm_torch.py:770-772 draws them, cached
    on `device` for repeated calls."""
    key = (int(n), int(m_probes), int(seed), dtype, str(device))
    Z = _PROBES.get(key)
    if Z is None:
        g = torch.Generator(device="cpu").manual_seed(seed)
        Z = (torch.randint(0, 2, (n, m_probes), generator=g, dtype=dtype) * 2.0 - 1.0).to(device)
        if len(_PROBES) >= 2:
            _PROBES.pop(next(iter(_PROBES)))
        _PROBES[key] = Z
    return Z


def slq_logdet(matvec, n, params, m_probes=20, lanczos_m=50, seed=0, dtype=torch.float64, device="cpu",
               batched=True):
    """Hutchinson + Lanczos-quadrature estimate of log det A(params), differentiable
    with respect to params (funm_torch.py:730-781).  The result lives on `device`."""
    from .imgp import ImgpPrecisionMatvec, _slq_logdet_fused

    params = tuple(params)
    dev = _slq.require_cuda()
    if isinstance(matvec, ImgpPrecisionMatvec) and batched and len(params) == 2:
        Z = _probes(n, m_probes, seed, matvec.dtype if dtype == matvec.dtype else dtype, matvec.device)
        if Z.dtype != matvec.dtype:
            Z = Z.to(matvec.dtype)
        return _slq_logdet_fused(matvec, Z, lanczos_m, *params).to(device)
    if batched:
        Z = _probes(n, m_probes, seed, dtype, device)
        return _SLQLogdetBatched.apply(matvec, Z, lanczos_m, *params)
    Z = _probes(n, m_probes, seed, dtype, device)
    total = torch.zeros((), dtype=dtype, device=device)
    for i in range(m_probes):
        total = total + funm_qform_op(matvec, Z[:, i], params, lanczos_m, "log")
    return total / m_probes


# ---------------------------------------------------------------------------
# Quadratic form with an operator-callable backward
# ---------------------------------------------------------------------------
class _FunmQFormKraemerOp(torch.autograd.Function):
    """q = z^T f(A) z with gradients for z and the operator's params
    (funm_torch.py:380-544)."""

    @staticmethod
    def forward(ctx, matvec, z, m, func, *params):
        _check_func(func)
        bs = _Basis(z.shape[0], 1, int(m), z.dtype, z.device)
        Zb, _, _ = _slq.to_block(z.detach(), bs.dev, z.dtype)
        with torch.no_grad():
            bs.run(Zb, lambda x: matvec(x, *params), vector=True)
        q, ga, gb, _ = _slq.small_side(bs.alpha, bs.beta, bs.znorm, func, 0, g_scale=1.0)
        ctx.bs, ctx.ga, ctx.gb, ctx.Zb, ctx.q = bs, ga, gb, Zb, q
        ctx.matvec = matvec
        ctx.save_for_backward(z, *params)
        return q[0].to(z.device, z.dtype)

    @staticmethod
    def backward(ctx, g_q):
        z, *params = ctx.saved_tensors
        bs = ctx.bs
        g_out = g_q.detach().to(bs.dev, torch.float64).reshape(1)
        gp, xi = _reverse_sweep(bs, ctx.matvec, tuple(params), ctx.ga, ctx.gb, g_out, vector=True,
                                need_xi0=ctx.needs_input_grad[1])
        g_z = None
        if xi is not None:
            # d q / d ||z|| = 2 q / ||z||
            g_zn = g_out * 2.0 * ctx.q / bs.znorm
            gZ = torch.empty_like(ctx.Zb)
            bs.rec.start_grad(xi, bs.V[0], ctx.Zb, bs.znorm, g_zn, gZ)
            g_z = gZ[:, 0].to(z.device, z.dtype)
        ctx.bs = None
        return (None, g_z, None, None, *_grads_like(gp, params))


def funm_qform_op(matvec, z, params, m, func="log"):
    """Differentiable z^T f(A) z with an operator-callable backward."""
    return _FunmQFormKraemerOp.apply(matvec, z, m, func, *tuple(params))


# ---------------------------------------------------------------------------
# f(A) v for a dense A
# ---------------------------------------------------------------------------
class _FunmApplyKraemer(torch.autograd.Function):
    """y = f(A) v by m Lanczos steps (no reorthogonalisation) with the Kraemer
    adjoint backward (funm_torch.py:254-367)."""

    @staticmethod
    def forward(ctx, A, v, m, func):
        _check_func(func)
        n = v.shape[0]
        m = int(m)
        bs = _Basis(n, 1, m, v.dtype, v.device)
        Ad = A.detach().to(bs.dev, v.dtype).contiguous()
        Zb, _, _ = _slq.to_block(v.detach(), bs.dev, v.dtype)

        def dense(lam_blk, out_blk):
            _slq.dense_matvec(Ad, lam_blk, out_blk, bs.ld, bs.ld)

        bs.rec.start(Zb, bs.V[0], bs.znorm)
        for j in range(m):
            dense(bs.V[j], bs.W)
            bs.rec.step(j, m, bs.W, bs.V[j], bs.V[j - 1] if j > 0 else None, bs.R, bs.V[j + 1], bs.alpha, bs.beta)
        u, _, _, _ = _slq.small_side(bs.alpha, bs.beta, None, func, 1)       # (1, m) = f(T) e1
        Vm = bs.V[:m, :, 0].to(torch.float64)                                 # (m, n)
        y = bs.znorm[0] * (u[0] @ Vm)
        ctx.bs, ctx.Ad, ctx.Zb, ctx.u, ctx.func, ctx.dense = bs, Ad, Zb, u, func, dense
        ctx.in_dev = (A.device, A.dtype, v.device, v.dtype)
        return y.to(v.device, v.dtype)

    @staticmethod
    def backward(ctx, g_y):
        bs, u = ctx.bs, ctx.u
        m, n = bs.m, bs.n
        gy = g_y.detach().to(bs.dev, torch.float64)
        Vm = bs.V[:m, :, 0].to(torch.float64)
        vn = bs.znorm[0]
        # small side: y = vn V u  ->  g_u = vn V^T g_y, g_vn = <g_y, V u>, g_V[:, j] = vn u_j g_y
        g_u = (vn * (Vm @ gy)).reshape(1, m).contiguous()
        g_vn = (gy @ (u[0] @ Vm)).reshape(1)
        _, ga, gb, _ = _slq.small_side(bs.alpha, bs.beta, None, ctx.func, 2, gu=g_u, g_scale=1.0)
        G, _, _ = _slq.to_block(gy.to(bs.dtype), bs.dev, bs.dtype)
        dcoef = (vn * u).contiguous()                                         # (1, m)
        gA = torch.zeros((n, n), dtype=torch.float64, device=bs.dev)

        def acc(lam_blk, x_blk):
            _slq.outer_accumulate(lam_blk, x_blk, bs.ld, gA)

        _, xi = _reverse_sweep(bs, None, (), ga, gb, None, vector=True, need_xi0=True, dcoef=dcoef, G=G,
                               on_lambda=acc, plam=ctx.dense)
        gZ = torch.empty_like(ctx.Zb)
        bs.rec.start_grad(xi, bs.V[0], ctx.Zb, bs.znorm, g_vn, gZ)
        a_dev, a_dt, v_dev, v_dt = ctx.in_dev
        ctx.bs = None
        return gA.to(a_dev, a_dt), gZ[:, 0].to(v_dev, v_dt), None, None


def funm_apply_kraemer(A: torch.Tensor, v: torch.Tensor, m: int, func: str = "log") -> torch.Tensor:
    """Differentiable f(A) v with the Kraemer adjoint backward (dense A)."""
    return _FunmApplyKraemer.apply(A, v, m, func)
