"""Matrix-free operators: eigsh of an operator known only through y = A x.

The reference accepts any device matvec through ``FunctionOperator``
(src/matvec_operator.cuh:149-163: ``void fn(const double* d_x, double* d_y,
int n, void* user_data)``), and scipy's ``eigsh`` accepts a
``scipy.sparse.linalg.LinearOperator``.  Both reach the C ABI entry point
``lg_eigsh_plan_create_op`` here:

* a ``scipy.sparse.linalg.LinearOperator`` (or any object with ``shape`` and
  ``matvec`` that is not a sparse matrix) runs on the host: the plan copies
  each Lanczos vector to pinned host memory, calls ``matvec`` on a float64
  numpy vector and copies the result back (``LG_OP_HOST``);
* a :class:`CudaOperator` wraps a torch function of a float64 CUDA vector; it
  runs on the plan's CUDA stream without any host wait (``LG_OP_STREAM``);
* :func:`raw_device_callback` hands the plan a function of two device
  pointers, the reference's contract (``LG_OP_DEVICE``).

The Krylov basis, the Gram-Schmidt passes, the restarts and the Ritz vectors
stay in the CUDA library; only y = A x is the caller's.  An exception raised by
the caller's function is kept, the product is filled with NaN so that the
solve stops, and the exception is raised again from ``solve``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native


class CudaOperator:
    """A symmetric n x n operator as a torch function on CUDA float64 vectors.

    ``matvec(x)`` receives an (n,) float64 tensor on ``device`` and returns
    A x as an (n,) tensor (any float dtype; it is copied into the plan's
    vector).  It runs inside ``torch.cuda.stream(...)`` of the plan's stream,
    so torch operations in it are ordered with the solver's kernels.
    """

    def __init__(self, n: int, matvec, device=None):
        import torch

        self.n = int(n)
        self.shape = (self.n, self.n)
        self.dtype = np.dtype(np.float64)
        self.matvec = matvec
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                    torch.cuda.current_device())

    def __repr__(self):
        return f"CudaOperator(n={self.n}, device={self.device})"


def is_operator(A) -> bool:
    """True for a LinearOperator-like object that is not a matrix."""
    import scipy.sparse as sp

    if isinstance(A, CudaOperator):
        return True
    if sp.issparse(A) or isinstance(A, np.ndarray):
        return False
    return hasattr(A, "matvec") and hasattr(A, "shape")


class _CudaView:
    """A raw device vector of n doubles, seen by torch through the CUDA array
    interface (no copy, no stream synchronisation)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f8", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class Callback:
    """The ctypes callback of one plan and the error it may have caught."""

    def __init__(self, A):
        self.error: BaseException | None = None
        if isinstance(A, CudaOperator):
            self.kind = _native.LG_OP_STREAM
            self.fn = None
            self.sfn = _native.MATVEC_STREAM_FN(self._make_stream(A))
        else:
            self.kind = _native.LG_OP_HOST
            self.fn = _native.MATVEC_FN(self._make_host(A))
            self.sfn = None

    def _make_host(self, A):
        def cb(x, y, n, user):
            try:
                xa = np.ctypeslib.as_array((C.c_double * n).from_address(x))
                ya = np.ctypeslib.as_array((C.c_double * n).from_address(y))
                out = np.asarray(A.matvec(xa.copy()), dtype=np.float64).reshape(-1)
                if out.shape[0] != n:
                    raise ValueError(f"matvec returned {out.shape[0]} values for n={n}")
                ya[:] = out
            except BaseException as exc:  # noqa: BLE001 - re-raised by solve()
                if self.error is None:
                    self.error = exc
                np.ctypeslib.as_array((C.c_double * n).from_address(y))[:] = np.nan
        return cb

    def _make_stream(self, A: CudaOperator):
        import torch

        views = {}

        def cb(x, y, n, user, stream):
            try:
                key = (x, y, n)
                if key not in views:
                    views[key] = (torch.as_tensor(_CudaView(x, n), device=A.device),
                                  torch.as_tensor(_CudaView(y, n), device=A.device))
                xt, yt = views[key]
                with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=A.device)):
                    out = A.matvec(xt)
                    if out.shape != (n,) and out.numel() == n:
                        out = out.reshape(n)
                    if out.shape != (n,):
                        raise ValueError(f"matvec returned shape {tuple(out.shape)} for n={n}")
                    yt.copy_(out)
            except BaseException as exc:  # noqa: BLE001 - re-raised by solve()
                if self.error is None:
                    self.error = exc
                with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=A.device)):
                    torch.as_tensor(_CudaView(y, n), device=A.device).fill_(float("nan"))
        return cb

    def create_plan(self, n: int, max_ncv: int):
        h = C.c_void_p()
        fn = C.cast(self.fn, C.c_void_p) if self.fn is not None else None
        sfn = C.cast(self.sfn, C.c_void_p) if self.sfn is not None else None
        _native.check(_native.lib.lg_eigsh_plan_create_op(C.byref(h), int(n), self.kind, fn, sfn, None,
                                                          int(max_ncv)))
        return h

    def raise_pending(self):
        if self.error is not None:
            exc, self.error = self.error, None
            raise exc


def raw_device_callback(fn):
    """Wrap a Python function ``fn(x_ptr, y_ptr, n)`` of two device pointers
    (ints) as an ``LG_OP_DEVICE`` callback: the reference's FunctionOperator
    contract, where the library waits for the whole device after each call."""

    class _Raw(Callback):
        def __init__(self):
            self.error = None
            self.kind = _native.LG_OP_DEVICE
            self.sfn = None

            def cb(x, y, n, user):
                try:
                    fn(int(x), int(y), int(n))
                except BaseException as exc:  # noqa: BLE001 - re-raised by solve()
                    if self.error is None:
                        self.error = exc
            self.fn = _native.MATVEC_FN(cb)

    return _Raw()
