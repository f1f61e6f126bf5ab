"""CPU (torch) restatement of the reference's stochastic Lanczos quadrature path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() to check
results, and by bench.py's cpu_baseline leg.  The product path never imports
it.  Pinned against golden vectors produced by the reference's own code
(tests/golden/make_golden.py).

Follows (reference file:line, python/gpu_eigsh/...):
  rademacher probes ............ funm_torch.py:770-773
  batched 3-term Lanczos ....... funm_torch.py:120-173
  SLQ forward .................. funm_torch.py:583-615
  SLQ backward (small side by
    autograd through eigh, then
    the Kraemer reverse sweep
    with an operator VJP) ...... funm_torch.py:617-727
  un-batched Lanczos ........... funm_torch.py:83-117
  funm_apply_kraemer ........... funm_torch.py:254-373
  funm_qform_op ................ funm_torch.py:380-564
  IMGP Laplacian cache ......... imgp.py:142-189
  L_sym matvec ................. imgp.py:192-207
  precision matvec ............. imgp.py:234-289
"""
from __future__ import annotations

import torch


def rademacher(n, m_probes, seed, dtype):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, 2, (n, m_probes), generator=g, dtype=dtype) * 2.0 - 1.0


def lanczos_batched(mv, Z, m):
    """B independent 3-term Lanczos runs, no reorthogonalisation."""
    zn = torch.linalg.vector_norm(Z, dim=0)
    V = [Z / zn]
    al, be = [], []
    prev = torch.zeros_like(V[0])
    bprev = torch.zeros(Z.shape[1], dtype=Z.dtype)
    for j in range(m):
        W = mv(V[j])
        a = (V[j] * W).sum(dim=0)
        R = W - a * V[j] - bprev * prev
        b = torch.linalg.vector_norm(R, dim=0)
        al.append(a)
        be.append(b)
        prev, bprev = V[j], b
        V.append(R / b)
    return torch.stack(V, dim=2), torch.stack(al, dim=1), torch.stack(be, dim=1), zn


def lanczos_single(mv, v, m):
    vn = torch.linalg.norm(v)
    V = [v / vn]
    al, be = [], []
    prev = torch.zeros_like(V[0])
    bprev = torch.zeros((), dtype=v.dtype)
    for j in range(m):
        w = mv(V[j])
        a = V[j] @ w
        r = w - a * V[j] - bprev * prev
        b = torch.linalg.norm(r)
        al.append(a)
        be.append(b)
        prev, bprev = V[j], b
        V.append(r / b)
    return torch.stack(V, dim=1), torch.stack(al), torch.stack(be), vn


def _tridiag_batched(a, bsub):
    B, m = a.shape
    T = torch.zeros(B, m, m, dtype=a.dtype)
    i = torch.arange(m)
    T[:, i, i] = a
    T[:, i[:-1], i[1:]] = bsub
    T[:, i[1:], i[:-1]] = bsub
    return T


def _quad_logdet(a, bsub, zn):
    Th, S = torch.linalg.eigh(_tridiag_batched(a, bsub))
    c = S[:, 0, :]
    return (zn * zn * (c * c * torch.log(Th)).sum(dim=1)).mean()


class _SLQ(torch.autograd.Function):
    @staticmethod
    def forward(ctx, matvec, Z, m, *params):
        with torch.no_grad():
            V, a, b, zn = lanczos_batched(lambda X: matvec(X, *params), Z, m)
            ld = _quad_logdet(a, b[:, :-1], zn)
        ctx.save_for_backward(Z, V, a, b, zn, *params)
        ctx.matvec, ctx.m = matvec, m
        return ld

    @staticmethod
    def backward(ctx, g_ld):
        Z, V, a, b, zn, *params = ctx.saved_tensors
        matvec, m = ctx.matvec, ctx.m
        n, B = Z.shape
        a_ = a.detach().clone().requires_grad_(True)
        bs_ = b[:, :-1].detach().clone().requires_grad_(True)
        with torch.enable_grad():
            ld = _quad_logdet(a_, bs_, zn)
            g_a, g_bs = torch.autograd.grad(ld, (a_, bs_), grad_outputs=g_ld)
        g_b = torch.cat([g_bs, torch.zeros(B, 1, dtype=Z.dtype)], dim=1)
        xi = torch.zeros(n, B, dtype=Z.dtype)
        lam_plus = torch.zeros(n, B, dtype=Z.dtype)
        grads = [torch.zeros_like(p) for p in params]
        pd = tuple(p.detach().clone().requires_grad_(True) for p in params)
        for j in range(m - 1, -1, -1):
            x, xp = V[:, :, j], V[:, :, j + 1]
            xd = xi / b[:, j]
            mu = g_b[:, j] - (lam_plus * x).sum(0) + (xp * xd).sum(0)
            nu = g_a[:, j] + (x * xd).sum(0)
            lam = -xd + mu * xp + nu * x
            with torch.enable_grad():
                out = matvec(x.detach(), *pd)
                gp = torch.autograd.grad(out, pd, grad_outputs=lam.detach(), allow_unused=True)
            for k, g in enumerate(gp):
                if g is not None:
                    grads[k] = grads[k] + g
            with torch.no_grad():
                Plam = matvec(lam, *params)
            xi = -Plam + a[:, j] * lam + b[:, j] * lam_plus - (b[:, j] * nu) * xp
            lam_plus = lam
        return (None, None, None, *grads)


def slq_logdet(matvec, n, params, m_probes=20, lanczos_m=50, seed=0, dtype=torch.float64):
    Z = rademacher(n, m_probes, seed, dtype)
    return _SLQ.apply(matvec, Z, lanczos_m, *params)


def _fn(theta, func):
    return {"log": torch.log, "exp": torch.exp, "sqrt": torch.sqrt, "inv": lambda t: 1.0 / t}[func](theta)


def _small_side(V, a, bsub, vn, func):
    m = a.shape[0]
    T = torch.diag(a)
    if m > 1:
        T = T + torch.diag(bsub, 1) + torch.diag(bsub, -1)
    Th, S = torch.linalg.eigh(T)
    c = S[0, :]
    return vn * (V @ (S @ (_fn(Th, func) * c)))


class _Kraemer(torch.autograd.Function):
    """y = f(A) v (dense A) with the Kraemer adjoint backward."""

    @staticmethod
    def forward(ctx, A, v, m, func):
        with torch.no_grad():
            V, a, b, vn = lanczos_single(lambda x: A @ x, v, m)
            y = _small_side(V[:, :m], a, b[:-1], vn, func)
        ctx.save_for_backward(A, v, V, a, b, vn)
        ctx.m, ctx.func = m, func
        return y

    @staticmethod
    def backward(ctx, g_y):
        A, v, V, a, b, vn = ctx.saved_tensors
        m, func = ctx.m, ctx.func
        n = v.shape[0]
        V_ = V[:, :m].detach().clone().requires_grad_(True)
        a_ = a.detach().clone().requires_grad_(True)
        b_ = b[:-1].detach().clone().requires_grad_(True)
        vn_ = vn.detach().clone().requires_grad_(True)
        with torch.enable_grad():
            y = _small_side(V_, a_, b_, vn_, func)
            gV, ga, gb, gvn = torch.autograd.grad(y, (V_, a_, b_, vn_), grad_outputs=g_y)
        gV = torch.cat([gV, torch.zeros(n, 1, dtype=v.dtype)], dim=1)
        gb = torch.cat([gb, torch.zeros(1, dtype=v.dtype)])
        xi = -gV[:, m].clone()
        lp = torch.zeros(n, dtype=v.dtype)
        gA = torch.zeros(n, n, dtype=v.dtype)
        for j in range(m - 1, -1, -1):
            x, xp = V[:, j], V[:, j + 1]
            xd = xi / b[j]
            mu = gb[j] - lp @ x + xp @ xd
            nu = ga[j] + x @ xd
            lam = -xd + mu * xp + nu * x
            gA = gA + torch.outer(lam, x)
            xi = -gV[:, j] - A @ lam + a[j] * lam + b[j] * lp - b[j] * nu * xp
            lp = lam
        v0 = V[:, 0]
        gv = ((xi @ v0) * v0 - xi) / vn + gvn * (v / vn)
        return gA, gv, None, None


def funm_apply_kraemer(A, v, m, func="log"):
    return _Kraemer.apply(A, v, m, func)


class _QForm(torch.autograd.Function):
    """z^T f(A) z with an operator-callable VJP (single probe)."""

    @staticmethod
    def forward(ctx, matvec, z, m, func, *params):
        with torch.no_grad():
            V, a, b, zn = lanczos_single(lambda x: matvec(x, *params), z, m)
            T = torch.diag(a) + torch.diag(b[:-1], 1) + torch.diag(b[:-1], -1)
            Th, S = torch.linalg.eigh(T)
            q = zn * zn * (S[0, :] ** 2 * _fn(Th, func)).sum()
        ctx.save_for_backward(z, V, a, b, zn, *params)
        ctx.matvec, ctx.m, ctx.func = matvec, m, func
        return q

    @staticmethod
    def backward(ctx, g_q):
        z, V, a, b, zn, *params = ctx.saved_tensors
        matvec, m, func = ctx.matvec, ctx.m, ctx.func
        n = z.shape[0]
        a_ = a.detach().clone().requires_grad_(True)
        b_ = b[:-1].detach().clone().requires_grad_(True)
        zn_ = zn.detach().clone().requires_grad_(True)
        with torch.enable_grad():
            T = torch.diag(a_) + torch.diag(b_, 1) + torch.diag(b_, -1)
            Th, S = torch.linalg.eigh(T)
            q = zn_ * zn_ * (S[0, :] ** 2 * _fn(Th, func)).sum()
            ga, gb, gzn = torch.autograd.grad(q, (a_, b_, zn_), grad_outputs=g_q)
        gb = torch.cat([gb, torch.zeros(1, dtype=z.dtype)])
        xi = torch.zeros(n, dtype=z.dtype)
        lp = torch.zeros(n, dtype=z.dtype)
        grads = [torch.zeros_like(p) for p in params]
        pd = tuple(p.detach().clone().requires_grad_(True) for p in params)
        for j in range(m - 1, -1, -1):
            x, xp = V[:, j], V[:, j + 1]
            xd = xi / b[j]
            mu = gb[j] - lp @ x + xp @ xd
            nu = ga[j] + x @ xd
            lam = -xd + mu * xp + nu * x
            with torch.enable_grad():
                out = matvec(x.detach(), *pd)
                gp = torch.autograd.grad(out, pd, grad_outputs=lam.detach(), allow_unused=True)
            for k, g in enumerate(gp):
                if g is not None:
                    grads[k] = grads[k] + g
            with torch.no_grad():
                Pl = matvec(lam, *params)
            xi = -Pl + a[j] * lam + b[j] * lp - b[j] * nu * xp
            lp = lam
        v0 = V[:, 0]
        gz = ((xi @ v0) * v0 - xi) / zn + gzn * (z / zn)
        return (None, gz, None, None, *grads)


def funm_qform_op(matvec, z, params, m, func="log"):
    return _QForm.apply(matvec, z, m, func, *params)


# ---- IMGP operator -----------------------------------------------------------

def laplacian_pieces(d2, idx, n, kappa, self_loops=True):
    """(diag (n,), triu (M,)) of the symmetric-normalised Laplacian with
    self-loops, as functions of the graph bandwidth kappa (autograd-able)."""
    k2 = kappa.square().squeeze()
    w = torch.exp(-d2 / (4 * k2))
    src, dst = idx[0], idx[1]
    du = (torch.ones if self_loops else torch.zeros)(n, dtype=d2.dtype)
    du = du.scatter_add(0, src, w).scatter_add(0, dst, w)
    adj = w / (du[src] * du[dst])
    deg = du.pow(-2) if self_loops else torch.zeros_like(du)
    deg = deg.scatter_add(0, src, adj).scatter_add(0, dst, adj)
    if self_loops:
        diag = (1.0 - du.pow(-2) / deg) / k2
    else:
        diag = torch.ones(n, dtype=d2.dtype) / k2
    ds = deg.sqrt()
    triu = adj / (ds[src] * ds[dst]) / k2
    return diag, triu


def lsym_matmul(X, diag, triu, idx):
    one = X.ndim == 1
    Xv = X.view(-1, 1) if one else X
    out = Xv * diag.view(-1, 1)
    out = out.index_add(0, idx[0], -triu.view(-1, 1) * Xv[idx[1]])
    out = out.index_add(0, idx[1], -triu.view(-1, 1) * Xv[idx[0]])
    return out.squeeze(-1) if one else out


def make_precision_matvec(d2, idx, n, nu, self_loops=True):
    cache = {"key": None, "val": None}

    def pieces(kappa):
        key = (id(kappa), kappa._version)
        if cache["key"] != key:
            cache["key"] = key
            cache["val"] = laplacian_pieces(d2, idx, n, kappa, self_loops)
        return cache["val"]

    def matvec(rhs, ell, kappa):
        diag, triu = pieces(kappa)
        s = ell.square().squeeze() / (2 * nu)
        out = rhs
        for _ in range(nu):
            out = (out + s * lsym_matmul(out, diag, triu, idx)) / s
        return out

    return matvec
