"""Device-pointer primitives of the Lanczos engine, for torch CUDA tensors.

``cgs2_orthogonalize(V, ncols, w)`` — two classical Gram-Schmidt passes of w
against the first ``ncols`` columns of the row-major basis V (the
reorthogonalisation step of every Lanczos step; the reference's
cgs_orthogonalize + dgks_reorth, src/lanczos_ops.cuh:113-192).
"""
from __future__ import annotations

from . import _native


def _stream_handle(t):
    import torch

    return torch.cuda.current_stream(t.device).cuda_stream


def cgs2_orthogonalize(V, ncols: int, w, r=None, coef=None, norms=None):
    """V: (n, ldv) float64 CUDA tensor, C-contiguous, ldv even; w: (n,) float64.

    Returns (r, coef, norms): r = (I - V V^T)^2 w restricted to the first
    ncols columns, coef = h1 + s (ncols,), norms = (||w||, ||r1||, ||r||).
    Runs on the current torch stream; asynchronous like any torch op."""
    import torch

    if V.dtype != torch.float64 or w.dtype != torch.float64 or not V.is_cuda or not w.is_cuda:
        raise TypeError("V and w must be float64 CUDA tensors")
    if not V.is_contiguous() or V.dim() != 2 or w.dim() != 1 or w.shape[0] != V.shape[0]:
        raise ValueError("V must be a contiguous (n, ldv) matrix and w a length-n vector")
    n, ldv = V.shape
    r = torch.empty_like(w) if r is None else r
    coef = torch.empty(ncols, dtype=torch.float64, device=V.device) if coef is None else coef
    norms = torch.empty(3, dtype=torch.float64, device=V.device) if norms is None else norms
    _native.check(_native.lib.lg_cgs2_orthogonalize(V.data_ptr(), int(ldv), int(n), int(ncols), w.data_ptr(),
                                                    r.data_ptr(), coef.data_ptr(), norms.data_ptr(),
                                                    _stream_handle(V)))
    return r, coef, norms
