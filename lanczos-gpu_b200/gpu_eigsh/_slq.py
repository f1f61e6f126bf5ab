"""Thin torch-side driver of the SLQ kernels in liblanczos_b200.so.

Owns nothing but buffers: blocks of probe vectors are torch CUDA tensors of
shape (k, n, ld) (row-major n x ld blocks, ld even), per-probe scalars are
fp64 tensors, and every call runs on the current torch stream of the block's
device.  All arithmetic happens in the library (include/lanczos_b200.h,
"stochastic Lanczos quadrature"); this module only checks shapes, allocates
and passes pointers.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native

_L = _native.lib


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return _native.LG_F32
    if dtype == torch.float64:
        return _native.LG_F64
    raise TypeError(f"the SLQ kernels compute in float32 or float64, got {dtype}")


def require_cuda() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("gpu_eigsh: a CUDA device is required (the SLQ path has no CPU implementation)")
    return torch.device("cuda", torch.cuda.current_device())


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ld_for(b: int, dtype: torch.dtype) -> int:
    """Row stride of a block of b probe columns: a multiple of 4 (fp32) or 2
    (fp64) elements, so that every lane's vector is one 16-byte access."""
    q = 4 if dtype == torch.float32 else 2
    return (b + q - 1) // q * q


def workspace(op: _native.SlqOp | None, B: int, ld: int, device: torch.device):
    nbytes = _L.lg_slq_workspace_bytes(C.byref(op) if op is not None else None, int(B), int(ld))
    if nbytes == 0:
        raise _native.LanczosError(_native.LG_ERR_INVALID, "invalid SLQ workspace request: " + _native.last_error())
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device), int(nbytes)


def blocks(k: int, n: int, ld: int, dtype: torch.dtype, device: torch.device, zero: bool = False):
    f = torch.zeros if zero else torch.empty
    return f((k, n, ld), dtype=dtype, device=device)


def to_block(X: torch.Tensor, device: torch.device, dtype: torch.dtype):
    """(n,) or (n, B) -> contiguous (n, ld) block on `device` (padding columns zero)."""
    X2 = X.reshape(-1, 1) if X.dim() == 1 else X
    n, B = X2.shape
    ld = ld_for(B, dtype)
    if ld == B and X2.is_contiguous() and X2.device == device and X2.dtype == dtype:
        return X2, B, ld
    out = torch.zeros((n, ld), dtype=dtype, device=device)
    out[:, :B] = X2
    return out, B, ld


def p(t) -> int | None:
    return None if t is None else t.data_ptr()


class Operator:
    """lg_slq_op over device arrays kept alive by this object."""

    def __init__(self, n, rowptr, col, offval, diag, doffval, ddiag, shift, power, dtype):
        self.keep = (rowptr, col, offval, diag, doffval, ddiag)
        self.s = _native.SlqOp(
            n=int(n), nnz=int(col.numel()), rowptr=p(rowptr), col=p(col), offval=p(offval), diag=p(diag),
            doffval=p(doffval), ddiag=p(ddiag), shift=float(shift), power=int(power), dtype=dtype_code(dtype))
        self.device = diag.device
        self.dtype = dtype

    @property
    def ref(self):
        return C.byref(self.s)

    def apply(self, X: torch.Tensor, B: int, ld: int) -> torch.Tensor:
        Y = torch.empty_like(X)
        ws, nb = workspace(self.s, B, ld, self.device)
        _native.check(_L.lg_slq_apply(self.ref, B, ld, p(X), p(Y), p(ws), nb, stream(self.device)))
        return Y

    def apply_vjp(self, X: torch.Tensor, G: torch.Tensor, B: int, ld: int):
        gX = torch.empty_like(X)
        gp = torch.empty(2, dtype=torch.float64, device=self.device)
        ws, nb = workspace(self.s, B, ld, self.device)
        _native.check(_L.lg_slq_apply_vjp(self.ref, B, ld, p(X), p(G), p(gX), p(gp), p(ws), nb,
                                          stream(self.device)))
        return gX, gp

    def forward(self, Z: torch.Tensor, B: int, ld: int, m: int):
        """Batched recurrence: V (m+1, n, ld), Y (m*(power-1), n, ld), alpha, beta (B, m), znorm (B)."""
        n = self.s.n
        V = blocks(m + 1, n, ld, self.dtype, self.device)
        Y = blocks(m * (self.s.power - 1), n, ld, self.dtype, self.device) if self.s.power > 1 else None
        alpha = torch.empty((B, m), dtype=torch.float64, device=self.device)
        beta = torch.empty((B, m), dtype=torch.float64, device=self.device)
        znorm = torch.empty(B, dtype=torch.float64, device=self.device)
        ws, nb = workspace(self.s, B, ld, self.device)
        _native.check(_L.lg_slq_forward(self.ref, B, m, ld, p(Z), p(V), p(Y), p(alpha), p(beta), p(znorm), p(ws),
                                        nb, stream(self.device)))
        return V, Y, alpha, beta, znorm

    def backward(self, V, Y, alpha, beta, g_alpha, g_beta, g_out, B: int, ld: int, m: int):
        gp = torch.empty(2, dtype=torch.float64, device=self.device)
        ws, nb = workspace(self.s, B, ld, self.device)
        _native.check(_L.lg_slq_backward(self.ref, B, m, ld, p(V), p(Y), p(alpha), p(beta), p(g_alpha),
                                         p(g_beta), p(g_out), p(gp), p(ws), nb, stream(self.device)))
        return gp


def small_side(alpha, beta, znorm, func: str, mode: int, gu=None, g_scale: float = 1.0):
    """Per-probe small side (see lg_slq_small_side).  alpha, beta: (B, m) fp64."""
    B, m = alpha.shape
    dev = alpha.device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = g_alpha = g_beta = None
    if mode == 0:
        out = torch.empty(B, dtype=torch.float64, device=dev)
    elif mode == 1:
        out = torch.empty((B, m), dtype=torch.float64, device=dev)
    if mode != 1:
        g_alpha = torch.empty((B, m), dtype=torch.float64, device=dev)
        g_beta = torch.empty((B, m), dtype=torch.float64, device=dev)
    ws, nb = workspace(None, B, 0, dev)
    _native.check(_L.lg_slq_small_side(B, m, _native.FUNCS[func], mode, p(alpha), p(beta), p(znorm), p(gu),
                                       float(g_scale), p(out), p(g_alpha), p(g_beta), p(status), p(ws), nb,
                                       stream(dev)))
    return out, g_alpha, g_beta, status


class BlockRecurrence:
    """Recurrence and reverse sweep around a caller-supplied product (lg_slq_block_*)."""

    def __init__(self, n: int, B: int, ld: int, dtype: torch.dtype, device: torch.device):
        self.n, self.B, self.ld, self.dtype, self.device = n, B, ld, dtype, device
        self.code = dtype_code(dtype)
        self.ws, self.nb = workspace(None, B, ld, device)

    def _args(self):
        return self.n, self.B, self.ld, self.code

    def start(self, Z, V0, znorm):
        _native.check(_L.lg_slq_block_start(*self._args(), p(Z), p(V0), p(znorm), p(self.ws), self.nb,
                                            stream(self.device)))

    def step(self, j, m, W, Vj, Vjm1, R, Vnext, alpha, beta):
        _native.check(_L.lg_slq_block_step(*self._args(), j, m, p(W), p(Vj), p(Vjm1), p(R), p(Vnext), p(alpha),
                                           p(beta), p(self.ws), self.nb, stream(self.device)))

    def lam(self, j, m, xi, xplus, xj, beta, g_alpha, g_beta, g_out, lam):
        _native.check(_L.lg_slq_block_lambda(*self._args(), j, m, p(xi), p(xplus), p(xj), p(beta), p(g_alpha),
                                             p(g_beta), p(g_out), p(lam), p(self.ws), self.nb,
                                             stream(self.device)))

    def xi(self, j, m, Plam, lam, lplus, xplus, xj, xjm1, alpha, beta, dcoef, G, xi):
        _native.check(_L.lg_slq_block_xi(*self._args(), j, m, p(Plam), p(lam), p(lplus), p(xplus), p(xj), p(xjm1),
                                         p(alpha), p(beta), p(dcoef), p(G), p(xi), p(self.ws), self.nb,
                                         stream(self.device)))

    def start_grad(self, xi, V0, Z, znorm, g_znorm, gZ):
        _native.check(_L.lg_slq_block_start_grad(*self._args(), p(xi), p(V0), p(Z), p(znorm), p(g_znorm), p(gZ),
                                                 p(self.ws), self.nb, stream(self.device)))


def dense_matvec(A: torch.Tensor, x: torch.Tensor, y: torch.Tensor, ldx: int, ldy: int):
    n = A.shape[0]
    _native.check(_L.lg_dense_matvec(n, dtype_code(A.dtype), p(A), p(x), ldx, p(y), ldy, stream(A.device)))


def outer_accumulate(lam: torch.Tensor, x: torch.Tensor, ld: int, gA: torch.Tensor):
    n = gA.shape[0]
    _native.check(_L.lg_outer_accumulate(n, dtype_code(lam.dtype), p(lam), p(x), ld, p(gA), stream(gA.device)))
