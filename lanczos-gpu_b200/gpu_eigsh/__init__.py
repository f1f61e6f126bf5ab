"""gpu_eigsh — B200-native Lanczos eigensolver and stochastic Lanczos quadrature.

Drop-in for the reference package of the same name:

* ``gpu_eigsh(A, k, ...)`` — k eigenpairs of a sparse symmetric matrix by
  implicitly restarted Lanczos on the GPU, with ``scipy.sparse.linalg.eigsh``
  semantics (``k, which, sigma, ncv, maxiter, tol, v0``).  The reference's
  positional order ``(A, k, ncv, maxiter, tol, which, sigma, cg_max_iters,
  cg_tol)`` (python/gpu_eigsh/__init__.py:141-142) is accepted unchanged;
  ``ncv=0`` means "automatic" as in the reference.
* ``gpu_eigsh.funm_torch`` — ``slq_logdet``, ``funm_apply_kraemer``,
  ``funm_qform_op`` (torch.autograd.Functions).
* ``gpu_eigsh.imgp`` — ``make_imgp_precision_matvec``.
* ``differentiable_eigsh`` — eigenpairs as a torch.autograd.Function with the
  implicit-differentiation backward (``gpu_eigsh.differentiable``).
* ``funm_apply`` / ``funm_qform`` — f(A) v and v^T f(A) v by m-step Lanczos
  quadrature (numpy in, numpy out).

All arithmetic runs in the CUDA library ``_lib/liblanczos_b200.so``; there is
no CPU fallback.
"""
from __future__ import annotations

import time

import numpy as np

from . import _native
from . import operators as _operators
from ._native import LanczosError
from .operators import CudaOperator

__all__ = ["gpu_eigsh", "EigshPlan", "CudaOperator", "LanczosError", "ArpackNoConvergence", "differentiable_eigsh",
           "funm_apply", "funm_qform"]

_FUNM_MSG = {-1: "unknown func", -2: "invalid eigenvalue for func", -3: "zero input vector",
             -4: "tridiag eigensolver failure"}


def _funm(A, v, m, func, mode, name):
    import scipy.sparse as sp

    if not sp.issparse(A):
        raise TypeError("A must be a scipy sparse matrix")
    if A.shape[0] != A.shape[1]:
        raise ValueError(f"Matrix must be square, got {A.shape}")
    n = A.shape[0]
    vv = np.ascontiguousarray(v, dtype=np.float64).reshape(-1)
    if vv.shape[0] != n:
        raise ValueError(f"v must have length {n}, got {vv.shape[0]}")
    code = _native.FUNCS.get(func)
    if code is None:
        raise RuntimeError(f"{name} failed: {_FUNM_MSG[-1]}")
    m = min(int(m), n)
    if m < 1 or m > 127:
        raise ValueError("m must be between 1 and 127 (the Lanczos depth of one plan)")
    y = np.zeros(n) if mode == 1 else None
    val = _native.C.c_double(0.0)
    ma = _native.C.c_int(0)
    with EigshPlan(A, max_ncv=m) as plan:
        _native.check(_native.lib.lg_eigsh_plan_funm(plan._plan, _native.ptr(vv), 0, m, code, mode,
                                                     _native.ptr(y) if y is not None else None,
                                                     _native.C.byref(val), _native.C.byref(ma)))
    rc = int(ma.value)
    if rc < 0:
        raise RuntimeError(f"{name} failed: {_FUNM_MSG.get(rc, rc)}")
    return (y if mode == 1 else float(val.value)), rc


def funm_apply(A, v, m=50, func="log"):
    """y ~ f(A) v by m-step Lanczos quadrature (f in log, exp, sqrt, inv).

    A: scipy sparse symmetric (n x n); v: (n,).  Returns (y, m_actual),
    m_actual < m when the Krylov space is exhausted.  Raises RuntimeError with
    the reference's messages (unknown func, invalid eigenvalue for func, zero
    input vector).  Same call as the reference's gpu_eigsh.funm_apply
    (python/gpu_eigsh/__init__.py:72-115); m <= 127 here.
    """
    return _funm(A, v, m, func, 1, "funm_apply")


def funm_qform(A, v, m=50, func="log"):
    """v^T f(A) v by m-step Lanczos quadrature; returns (value, m_actual)."""
    return _funm(A, v, m, func, 0, "funm_qform")


def differentiable_eigsh(*args, **kwargs):
    """See gpu_eigsh.differentiable.differentiable_eigsh (imported on first use:
    it needs torch)."""
    from .differentiable import differentiable_eigsh as _impl

    return _impl(*args, **kwargs)

try:  # raise scipy's own exception type so existing handlers keep working
    from scipy.sparse.linalg import ArpackNoConvergence
except Exception:  # pragma: no cover - scipy is a dependency of the API
    class ArpackNoConvergence(RuntimeError):
        def __init__(self, msg, eigenvalues, eigenvectors):
            super().__init__(msg)
            self.eigenvalues = eigenvalues
            self.eigenvectors = eigenvectors


def _as_csr(A):
    """scipy sparse / dense ndarray -> (n, indptr int32, indices int32, data float64)."""
    import scipy.sparse as sp

    if sp.issparse(A):
        M = sp.csr_matrix(A, dtype=np.float64)
    elif isinstance(A, np.ndarray) and A.ndim == 2:
        M = sp.csr_matrix(np.asarray(A, dtype=np.float64))
    else:
        raise TypeError("A must be a scipy sparse matrix or a 2-D numpy array")
    if M.shape[0] != M.shape[1]:
        raise ValueError(f"Matrix must be square, got {M.shape}")
    # duplicate or unsorted entries need no pass here: the sparse products sum
    # every stored entry, which is the matrix scipy means
    indptr = np.ascontiguousarray(M.indptr, dtype=np.int32)
    indices = np.ascontiguousarray(M.indices, dtype=np.int32)
    data = np.ascontiguousarray(M.data, dtype=np.float64)
    return M.shape[0], indptr, indices, data


def _sync_caller_stream():
    """Device pointers handed to the library are read on the library's own
    non-blocking stream, which does not wait for the caller's: finish the
    work queued on torch's current stream first (a no-op without torch or
    without CUDA)."""
    import sys

    torch = sys.modules.get("torch")
    if torch is not None and torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.current_stream().synchronize()


def _default_ncv(n: int, k: int) -> int:
    # scipy.sparse.linalg._eigen.arpack.choose_ncv: max(2k+1, 20), capped at n
    return min(n, max(2 * k + 1, 20))


def _reorder_flag(reorder) -> int:
    if reorder is None or reorder is False:
        return 0
    if reorder is True or reorder in ("cm", "bfs"):
        return _native.LG_PLAN_REORDER_BFS
    if reorder == "degree":
        return _native.LG_PLAN_REORDER_DEGREE
    raise ValueError(f"reorder must be a bool, 'cm' or 'degree', got {reorder!r}")


class EigshPlan:
    """A matrix resident on the GPU plus the solver workspace.

    Reusing a plan skips the CSR upload and all device allocations, which is
    what a caller solving repeatedly on one matrix wants.  ``solve`` takes the
    same keywords as :func:`gpu_eigsh`.  ``reorder=True`` (or ``"cm"``)
    renumbers the rows inside the plan in Cuthill-McKee order
    (LG_PLAN_REORDER_BFS) for locality of the sparse product of mesh-like and
    kNN graphs; ``reorder="degree"`` renumbers them by descending row length
    (LG_PLAN_REORDER_DEGREE), which packs the hubs of a power-law graph
    together; v0, eigenvectors and ``matvec_device`` keep the caller's
    numbering.  ``cgs2_inline=True`` keeps both Gram-Schmidt passes inside
    every Lanczos step (LG_PLAN_CGS2_INLINE) instead of delaying the second
    pass into the next step's stream of the basis (same results to rounding).
    """

    def __init__(self, A, max_ncv: int = 127, mixed: bool = False, device_csr=None, comm=None, n_global=None,
                 reorder=False, cgs2_inline: bool = False, callback=None):
        self._plan = None
        self._cb = None
        if callback is not None or (A is not None and device_csr is None and _operators.is_operator(A)):
            # matrix-free: A is a LinearOperator / CudaOperator (or a raw
            # device callback with A giving the size)
            if mixed or reorder or comm is not None:
                raise ValueError("mixed, reorder and comm need a sparse matrix, not an operator")
            n = int(A.shape[0]) if hasattr(A, "shape") else int(A)
            if hasattr(A, "shape") and (len(A.shape) != 2 or A.shape[0] != A.shape[1]):
                raise ValueError(f"operator must be square, got shape {A.shape}")
            self._cb = callback if callback is not None else _operators.Callback(A)
            self._plan = self._cb.create_plan(n, max_ncv)
            self.n, self.nnz, self.mixed, self.max_ncv = n, 0, False, int(max_ncv)
            self.last_info = {}
            return
        flags = _reorder_flag(reorder) | (_native.LG_PLAN_CGS2_INLINE if cgs2_inline else 0)
        if reorder and comm is not None:
            raise ValueError("reorder a partitioned matrix before splitting it (gpu_eigsh.ordering)")
        if cgs2_inline and comm is not None:
            raise ValueError("cgs2_inline is a single-GPU plan option")
        h = _native.C.c_void_p()
        if device_csr is not None:
            # the library copies the arrays on its own stream: work still queued
            # on the caller's stream (the kernels that produced them) must be done
            _sync_caller_stream()
        if comm is not None:
            # row-partitioned: device_csr holds this rank's rows (global column indices)
            n, nnz, rp, ci, vals = device_csr
            rc = _native.lib.lg_eigsh_plan_create_dist(_native.C.byref(h), comm.handle, int(n_global), int(n),
                                                       int(nnz), int(rp), int(ci), int(vals), 1, int(max_ncv),
                                                       int(bool(mixed)))
        elif device_csr is not None:
            n, nnz, rp, ci, vals = device_csr
            rc = _native.lib.lg_eigsh_plan_create_ex(_native.C.byref(h), int(n), int(nnz), int(rp), int(ci),
                                                     int(vals), 1, int(max_ncv), int(bool(mixed)), flags)
        else:
            n, indptr, indices, data = _as_csr(A)
            nnz = data.shape[0]
            self._host = (indptr, indices, data)
            rc = _native.lib.lg_eigsh_plan_create_ex(_native.C.byref(h), n, nnz, _native.ptr(indptr),
                                                     _native.ptr(indices), _native.ptr(data), 0, int(max_ncv),
                                                     int(bool(mixed)), flags)
        _native.check(rc)
        self._plan = h
        self.n = int(n)
        self.nnz = int(nnz)
        self.mixed = bool(mixed)
        self.max_ncv = int(max_ncv)
        self.last_info: dict = {}

    def close(self):
        if self._plan is not None and self._plan.value:
            _native.lib.lg_eigsh_plan_destroy(self._plan)
        self._plan = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def factorize(self, v0, m):
        """m Lanczos steps (no restart) from v0; returns (alpha (m,), beta (m+1,))."""
        v0a = np.ascontiguousarray(np.asarray(v0, dtype=np.float64).reshape(-1))
        if v0a.shape[0] != self.n:
            raise ValueError("v0 has the wrong length")
        a = np.zeros(int(m))
        b = np.zeros(int(m) + 1)
        P = _native.C.POINTER(_native.C.c_double)
        rc = _native.lib.lg_eigsh_plan_factorize(self._plan, v0a.ctypes.data_as(P), int(m), a.ctypes.data_as(P),
                                                 b.ctypes.data_as(P))
        if self._cb is not None:
            self._cb.raise_pending()
        _native.check(rc)
        return a, b

    def matvec_device(self, x_ptr: int, y_ptr: int):
        """y = A x on device buffers (raw CUDA pointers, n doubles each)."""
        _sync_caller_stream()
        _native.check(_native.lib.lg_eigsh_plan_matvec(self._plan, int(x_ptr), int(y_ptr)))
        if self._cb is not None:
            self._cb.raise_pending()

    def solve(self, k=6, ncv=None, maxiter=None, tol=0.0, which="LM", sigma=None, cg_max_iters=None,
              cg_tol=1e-12, *, v0=None, return_eigenvectors=True, max_steps=None, seed=42,
              evecs_out=None, v0_device=None, evecs_layout="rowmajor", raise_noconv=True, profile=False):
        n = self.n
        k = int(k)
        if k <= 0:
            raise ValueError("k must be greater than 0.")
        if k >= n:
            raise ValueError(f"k must be less than ndim(A), k={k}")
        which = str(which).upper()
        if which not in _native.WHICH:
            raise ValueError("which must be one of LM SM LA SA BE")
        ncv_eff = _default_ncv(n, k) if (ncv is None or int(ncv) <= 0) else min(int(ncv), n)
        if ncv_eff <= k or ncv_eff > n:
            raise ValueError(f"ncv must be k<ncv<=n, ncv={ncv_eff}")
        if ncv_eff > self.max_ncv:
            raise ValueError(f"ncv={ncv_eff} exceeds this plan's max_ncv={self.max_ncv}")
        o = _native.EigshOpts()
        _native.lib.lg_eigsh_opts_default(_native.C.byref(o))
        o.k = k
        o.ncv = ncv_eff
        o.maxiter = 0 if maxiter is None else int(maxiter)
        if maxiter is not None and int(maxiter) <= 0:
            raise ValueError(f"maxiter must be positive, maxiter={maxiter}")
        o.max_steps = 0 if max_steps is None else int(max_steps)
        o.tol = float(tol) if tol is not None else 0.0
        o.which = _native.WHICH[which]
        o.use_sigma = 0 if sigma is None else 1
        o.sigma = 0.0 if sigma is None else float(sigma)
        o.cg_max_iters = 0 if cg_max_iters is None else int(cg_max_iters)
        o.cg_tol = float(cg_tol)
        o.mixed = int(self.mixed)
        o.seed = int(seed) & ((1 << 64) - 1)
        o.return_vectors = int(bool(return_eigenvectors))
        o.evecs_rowmajor = 1 if evecs_layout == "rowmajor" else 0
        o.profile = int(bool(profile))

        v0p = 0
        io_dev = 0
        if v0_device is not None:
            v0p, io_dev = int(v0_device), 1
        elif v0 is not None:
            v0a = np.ascontiguousarray(np.asarray(v0, dtype=np.float64).reshape(-1))
            if v0a.shape[0] != n:
                raise ValueError(f"v0 must have length {n}, got {v0a.shape[0]}")
            if not np.any(v0a):
                raise ValueError("v0 must not be the zero vector")
            v0p = _native.ptr(v0a)
        evals = np.zeros(k, dtype=np.float64)
        evecs = None
        evp = 0
        if return_eigenvectors:
            if evecs_out is not None:
                evp, io_dev = int(evecs_out), 1
            else:
                if io_dev:
                    raise ValueError("v0_device requires evecs_out (device pointer)")
                shape = (n, k) if evecs_layout == "rowmajor" else (k, n)
                evecs = np.zeros(shape, dtype=np.float64)
                evp = _native.ptr(evecs)
        info = _native.EigshInfo()
        if io_dev:
            _sync_caller_stream()   # v0 / the output buffer may come from the caller's queued work
        rc = _native.lib.lg_eigsh_plan_run(self._plan, _native.C.byref(o), v0p or None,
                                           evals.ctypes.data_as(_native.C.POINTER(_native.C.c_double)),
                                           evp or None, io_dev, _native.C.byref(info))
        self.last_info = info.as_dict()
        if self._cb is not None:
            self._cb.raise_pending()   # an exception of the caller's matvec comes first
        if rc == _native.LG_ERR_CG_NOCONV:
            raise LanczosError(rc, _native.last_error() + "; increase cg_max_iters or cg_tol")
        _native.check(rc)
        if evecs is not None and evecs_layout != "rowmajor":
            evecs = evecs.T
        if rc == _native.LG_NOCONV and raise_noconv:
            nconv = info.nconv
            msg = (f"ARPACK error -1: No convergence ({info.restarts} iterations, "
                   f"{nconv}/{k} eigenvectors converged)")
            raise ArpackNoConvergence(msg, evals, evecs)
        if return_eigenvectors:
            return evals, evecs
        return evals


def gpu_eigsh(A, k=6, ncv=None, maxiter=None, tol=0, which="LM", sigma=None, cg_max_iters=None,
              cg_tol=1e-12, *, v0=None, return_eigenvectors=True, mixed=False, max_steps=None, seed=42,
              return_info=False, M=None, mode="normal", reorder=False):
    """Compute k eigenvalues (and eigenvectors) of a sparse symmetric matrix on the GPU.

    Semantics follow ``scipy.sparse.linalg.eigsh``.  ``A`` is a scipy sparse
    matrix or dense array (uploaded as CSR), a
    ``scipy.sparse.linalg.LinearOperator`` (its ``matvec`` runs on the host,
    once per Lanczos step), or a :class:`CudaOperator` (a torch function of a
    CUDA vector, run on the solver's stream): the reference's
    FunctionOperator (src/matvec_operator.cuh:149-163).

    k : number of eigenpairs (1 <= k < n).
    ncv : Lanczos basis size; None or 0 -> min(n, max(2k+1, 20)).
    maxiter : maximum number of implicit restarts (ARPACK iterations);
        None -> 10 n.  ``max_steps`` additionally bounds the Lanczos steps
        (the reference's meaning of ``maxiter``).
    tol : relative accuracy of the Ritz values; 0 -> machine precision.
    which : 'LM', 'SM', 'LA', 'SA' or 'BE'.
    sigma : shift-invert about sigma: Lanczos on (A - sigma I)^-1 with an
        inner CG solve (``cg_max_iters``, ``cg_tol``); ``which`` then refers
        to the transformed eigenvalues (default 'LM' = nearest sigma).
        CG requires A - sigma I to be definite.
    v0 : starting vector (length n); None -> a seeded uniform random vector.
    mixed : fp32 matrix values with fp64 accumulation and fp64 basis.
    reorder : renumber the rows inside the solver for locality of the sparse
        product: True or 'cm' (Cuthill-McKee, mesh-like and kNN graphs) or
        'degree' (descending row length, power-law graphs); see EigshPlan.
        Results keep the caller's order.

    Returns ``(w, v)`` with ``w`` ascending and ``v`` of shape (n, k), or ``w``
    alone when ``return_eigenvectors=False``.  Raises scipy's
    ``ArpackNoConvergence`` (carrying the converged pairs) when maxiter is
    exhausted, and ``LanczosError`` for device-side failures.
    """
    if M is not None or mode != "normal":
        raise NotImplementedError("generalized problems (M) and non-normal shift-invert modes are not supported")
    if _operators.is_operator(A):
        if sigma is not None:
            raise NotImplementedError("shift-invert needs a sparse matrix (its inner CG multiplies by A); "
                                      "an operator has no such form")
        if mixed or reorder:
            raise ValueError("mixed and reorder need a sparse matrix, not an operator")
    n = A.shape[0]
    if k is not None and int(k) >= n:
        import scipy.sparse as sp
        if sp.issparse(A):
            raise TypeError("Cannot use scipy.linalg.eigh for sparse A with k >= N. "
                            "Use scipy.linalg.eigh(A.toarray()) or reduce k.")
    ncv_eff = _default_ncv(n, int(k)) if (ncv is None or int(ncv) <= 0) else min(int(ncv), n)
    t0 = time.perf_counter()
    plan = EigshPlan(A, max_ncv=max(ncv_eff, 2), mixed=mixed, reorder=reorder)
    t1 = time.perf_counter()
    try:
        try:
            out = plan.solve(k=k, ncv=ncv_eff, maxiter=maxiter, tol=tol, which=which, sigma=sigma,
                             cg_max_iters=cg_max_iters, cg_tol=cg_tol, v0=v0,
                             return_eigenvectors=return_eigenvectors, max_steps=max_steps, seed=seed)
        except ArpackNoConvergence as exc:
            exc.info = plan.last_info
            raise
        t2 = time.perf_counter()
    finally:
        plan.close()
    if return_info:
        info = dict(plan.last_info)
        # host wall time of the three phases: plan (CSR upload and checks,
        # workspace), solve (v0 up, iterations, eigenvectors down), close
        info["host_ms"] = {"plan": 1e3 * (t1 - t0), "solve": 1e3 * (t2 - t1),
                           "close": 1e3 * (time.perf_counter() - t2)}
        return out, info
    return out
