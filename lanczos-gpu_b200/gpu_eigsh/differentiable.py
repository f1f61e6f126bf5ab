"""Differentiable sparse eigendecomposition (torch.autograd) on the GPU.

Drop-in for the reference's python/gpu_eigsh/differentiable.py:

    differentiable_eigsh(A, k=20, ncv=0, maxiter=3000, tol=1e-12, sigma=None,
                         cg_max_iters=500, cg_tol=1e-10) -> (eigenvalues, eigenvectors)

A is a torch sparse CSR (or COO) tensor whose values may require grad; the
gradients flow back to A's stored values.  Forward: the k smallest-algebraic
eigenpairs by the implicitly restarted Lanczos engine (``maxiter`` = Lanczos
step budget, as the reference's compute_eigsh), or with ``sigma`` the k
nearest sigma by shift-invert; eigenvalues ascending, eigenvectors n x k.  As
in the reference, a solve that ends at the step budget returns the current
Ritz pairs without raising.

Backward (implicit differentiation, Xie et al. 2020, as the reference's
compute_adjoint_eigsh, python/gpu_eigsh/_cuda_eigsh.cu:183-326): for every pair
i, xi_i solves (A - lambda_i I) xi_i = (I - X X^T) dL/dx_i orthogonally to the
k computed eigenvectors X, and

    dL/dA[r, c] = sum_i (dL/dlambda_i x_i[r] - xi_i[r]) x_i[c]   (stored entries).

The k systems run as one block CG on the device (lg_eigsh_adjoint) instead of
the reference's k sequential solves with a host-side accumulation; the
gradient is formed on the device over the sparsity pattern.  Like the
reference, the deflation drops the coupling between computed eigenvectors, so
eigenvector gradients are exact only where the loss gradient is orthogonal to
the other computed eigenvectors (always for eigenvalue-only losses, where this
reduces to the Hellmann-Feynman term x_i x_i^T).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native

__all__ = ["differentiable_eigsh"]


def _cuda_device(t: torch.Tensor) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("differentiable_eigsh needs a CUDA device (there is no CPU fallback)")
    return t.device if t.is_cuda else torch.device("cuda", torch.cuda.current_device())


# From this many rows on, the matrix is renumbered (Cuthill-McKee) for the
# solve and the backward: the block of k gathered columns (n x k doubles) no
# longer fits in L2, and in a random vertex order every gather of the sparse
# products would go to DRAM.
REORDER_MIN_ROWS = 1 << 16


class _DifferentiableEigsh(torch.autograd.Function):
    @staticmethod
    def forward(ctx, values, crow, col, n, k, ncv, maxiter, tol, sigma, cg_max_iters, cg_tol):
        from . import EigshPlan

        dev = _cuda_device(values)
        rp = crow.detach().to(dev, torch.int32).contiguous()
        ci = col.detach().to(dev, torch.int32).contiguous()
        va = values.detach().to(dev, torch.float64).contiguous()
        nnz = int(ci.numel())
        perm = order = pos = None
        if int(n) >= REORDER_MIN_ROWS and nnz > 0:
            # the renumbering walks the graph: check the CSR first (the plan
            # checks it again on its own)
            if (rp.numel() != int(n) + 1 or int(rp[0]) != 0 or int(rp[-1]) != nnz or bool((rp[1:] < rp[:-1]).any())
                    or int(ci.min()) < 0 or int(ci.max()) >= int(n)):
                raise ValueError("malformed CSR (row pointers or column indices)")
            from .ordering import cm_order, permute_symmetric

            with torch.cuda.device(dev):
                perm = cm_order(rp, ci)
                rp, ci, va, pos, order = permute_symmetric(rp, ci, va, perm, return_order=True)
        with torch.cuda.device(dev):
            torch.cuda.current_stream(dev).synchronize()   # the plan copies the CSR on its own stream
            plan = EigshPlan(None, max_ncv=max(int(ncv), 2),
                             device_csr=(int(n), nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr()))
            try:
                Y = torch.empty((int(n), int(k)), dtype=torch.float64, device=dev)
                kw = dict(k=int(k), ncv=int(ncv), tol=float(tol), max_steps=int(maxiter), evecs_out=Y.data_ptr(),
                          raise_noconv=False)
                if sigma is None:
                    w, _ = plan.solve(which="SA", **kw)
                else:
                    w, _ = plan.solve(which="LM", sigma=float(sigma), cg_max_iters=int(cg_max_iters),
                                      cg_tol=float(cg_tol), **kw)
            finally:
                plan.close()
        evals = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
        ctx.save_for_backward(evals, Y, va, rp, ci)
        ctx.perm, ctx.order = perm, order
        ctx.n, ctx.k, ctx.cg = int(n), int(k), (int(cg_max_iters), float(cg_tol))
        ctx.vdev, ctx.vdtype = values.device, values.dtype
        Yc = Y if pos is None else Y.index_select(0, pos)   # rows back in the caller's numbering
        return evals.to(values.device), Yc.to(values.device)

    @staticmethod
    def backward(ctx, g_evals, g_evecs):
        evals, Y, va, rp, ci = ctx.saved_tensors
        dev = va.device
        n, k = ctx.n, ctx.k
        ge = None if g_evals is None else g_evals.detach().to(dev, torch.float64).contiguous()
        gv = None if g_evecs is None else g_evecs.detach().to(dev, torch.float64)
        if gv is not None and ctx.perm is not None:
            gv = gv.index_select(0, ctx.perm)   # into the solve's numbering
        gv = None if gv is None else gv.contiguous()
        grad = torch.empty(va.numel(), dtype=torch.float64, device=dev)
        iters = (C.c_int * k)()
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            _native.check(_native.lib.lg_eigsh_adjoint(
                n, int(va.numel()), rp.data_ptr(), ci.data_ptr(), va.data_ptr(), k, evals.data_ptr(), Y.data_ptr(),
                ge.data_ptr() if ge is not None else None, gv.data_ptr() if gv is not None else None,
                grad.data_ptr(), ctx.cg[0], ctx.cg[1], iters, stream))
        ctx.cg_iters = list(iters)
        if ctx.order is not None:   # entries back in the caller's storage order
            g2 = torch.empty_like(grad)
            g2[ctx.order] = grad
            grad = g2
        return (grad.to(ctx.vdev, ctx.vdtype), None, None, None, None, None, None, None, None, None, None)


def _direct_values(A: torch.Tensor) -> torch.Tensor:
    """A.values(), connected to the autograd graph past the sparse constructor.

    torch's backward of torch.sparse_csr_tensor(crow, col, values) forms the
    gradient of A densely (n x n: 8 TB at n = 1e6) before sampling it at the
    stored entries.  When A comes straight from that constructor, its saved
    `values` input is returned instead, so the gradient flows to it entry by
    entry; otherwise (or if this torch build names things differently) A.values().
    """
    vals = A.values()
    node = A.grad_fn
    if node is not None and type(node).__name__.startswith("SparseCompressedTensorBackward"):
        try:
            saved = node._saved_values
        except (AttributeError, RuntimeError):
            return vals
        if isinstance(saved, torch.Tensor) and saved.shape == vals.shape and saved.data_ptr() == vals.data_ptr():
            return saved
    return vals


def differentiable_eigsh(A, k=20, ncv=0, maxiter=3000, tol=1e-12, sigma=None, cg_max_iters=500, cg_tol=1e-10):
    """k eigenpairs of a symmetric sparse matrix with gradients to its values.

    A : torch sparse CSR or COO tensor (values may require grad), or a scipy
        sparse matrix (no gradients; the pairs come back as torch tensors).
    k, ncv, maxiter, tol, sigma, cg_max_iters, cg_tol : as the reference
        (ncv = 0 -> min(3k, n - 1) for torch input; maxiter counts Lanczos
        steps; the CG settings drive the backward and the shift-invert solve).
    Returns (eigenvalues (k,), eigenvectors (n, k)) float64 tensors on the
    device of A's values, eigenvalues ascending.
    """
    if isinstance(A, torch.Tensor):
        if A.layout == torch.sparse_csr:
            crow, col, values = A.crow_indices(), A.col_indices(), _direct_values(A)
        elif A.is_sparse:
            Acsr = A.coalesce().to_sparse_csr()
            crow, col, values = Acsr.crow_indices(), Acsr.col_indices(), Acsr.values()
        else:
            raise TypeError("A must be a sparse torch tensor (CSR or COO)")
        n = int(A.shape[0])
        if A.shape[0] != A.shape[1]:
            raise ValueError("A must be square")
        if ncv == 0:
            ncv = min(3 * int(k), n - 1)
        return _DifferentiableEigsh.apply(values, crow, col, n, int(k), int(ncv), int(maxiter), float(tol), sigma,
                                          int(cg_max_iters), float(cg_tol))
    # scipy sparse: no autograd
    from . import gpu_eigsh

    if sigma is None:
        w, V = gpu_eigsh(A, k=k, ncv=ncv, which="SA", tol=tol, max_steps=maxiter)
    else:
        w, V = gpu_eigsh(A, k=k, ncv=ncv, sigma=sigma, tol=tol, max_steps=maxiter, cg_max_iters=cg_max_iters,
                         cg_tol=cg_tol)
    return torch.from_numpy(w), torch.from_numpy(V)
