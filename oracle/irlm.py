"""Python wrapper of the CPU IRLM oracle (irlm_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, by __graft_entry__.smoke() to check
results and by bench.py's cpu_baseline / --impl reference leg.  The product
path (gpu_eigsh) never imports this module.

Also exposes ``arpack_eigsh`` — scipy.sparse.linalg.eigsh (ARPACK), the ground
truth the reference itself checks against (tests/test_gradient.py:59-81,
benchmark/scipy_reference.py:30).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

from .build_oracle import build as _build

_WHICH = {"LM": 0, "SM": 1, "LA": 2, "SA": 3, "BE": 4}
_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build()
        L = C.CDLL(str(path))
        PD, PI, PLL = C.POINTER(C.c_double), C.POINTER(C.c_int), C.POINTER(C.c_longlong)
        L.oracle_irlm.restype = C.c_int
        L.oracle_irlm.argtypes = [C.c_int, PI, PI, PD, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int,
                                  C.c_longlong, PD, C.c_uint64, C.c_int, PD, PD, PLL, PD, PD]
        L.oracle_lanczos_steps.restype = C.c_longlong
        L.oracle_lanczos_steps.argtypes = [C.c_int, PI, PI, PD, C.c_int, PD, C.c_int, PD, PD]
        L.oracle_num_threads.restype = C.c_int
        L.oracle_set_num_threads.restype = C.c_int
        L.oracle_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _csr(A):
    import scipy.sparse as sp

    M = sp.csr_matrix(A, dtype=np.float64)
    M.sum_duplicates()
    return (M.shape[0], np.ascontiguousarray(M.indptr, dtype=np.int32),
            np.ascontiguousarray(M.indices, dtype=np.int32), np.ascontiguousarray(M.data, dtype=np.float64))


def _p(a, t):
    return None if a is None else a.ctypes.data_as(C.POINTER(t))


def oracle_eigsh(A, k, ncv=None, which="LM", tol=0.0, maxiter=None, max_steps=0, v0=None, seed=42,
                 cgs2=True, return_eigenvectors=True, return_factorization=False):
    """IRLM on the CPU.  Returns (evals ascending, evecs (n,k)), info dict."""
    n, ip, ix, dv = _csr(A)
    m = min(n, max(2 * k + 1, 20)) if not ncv else int(ncv)
    ev = np.zeros(k)
    vec = np.zeros((k, n)) if return_eigenvectors else None
    info = np.zeros(5, dtype=np.int64)
    a0 = np.zeros(m)
    b0 = np.zeros(m + 1)
    v0a = None if v0 is None else np.ascontiguousarray(v0, dtype=np.float64)
    rc = lib().oracle_irlm(n, _p(ip, C.c_int), _p(ix, C.c_int), _p(dv, C.c_double), int(k), int(m),
                           _WHICH[which.upper()], float(tol), int(maxiter or 0), int(max_steps or 0),
                           _p(v0a, C.c_double), int(seed), int(bool(cgs2)), _p(ev, C.c_double),
                           _p(vec, C.c_double), info.ctypes.data_as(C.POINTER(C.c_longlong)),
                           _p(a0, C.c_double), _p(b0, C.c_double))
    if rc < 0:
        raise RuntimeError(f"oracle_irlm failed: {rc}")
    out = {"converged": rc == 0, "nconv": int(info[0]), "restarts": int(info[1]), "steps": int(info[2]),
           "reorth_passes": int(info[3]), "breakdowns": int(info[4])}
    if return_factorization:
        out["alpha0"] = a0
        out["beta0"] = b0
    return (ev, None if vec is None else vec.T.copy()), out


def oracle_lanczos_steps(A, m, v0, cgs2=True):
    """m Lanczos steps from v0 (no restart); returns (alpha (m,), beta (m+1,))."""
    n, ip, ix, dv = _csr(A)
    a = np.zeros(m)
    b = np.zeros(m + 1)
    v0a = np.ascontiguousarray(v0, dtype=np.float64)
    lib().oracle_lanczos_steps(n, _p(ip, C.c_int), _p(ix, C.c_int), _p(dv, C.c_double), int(m),
                               _p(v0a, C.c_double), int(bool(cgs2)), _p(a, C.c_double), _p(b, C.c_double))
    return a, b


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def host_cores() -> int:
    """Cores this process may run on (its affinity mask), not what a launcher
    put into OMP_NUM_THREADS."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def set_num_threads(nth: int | None = None) -> int:
    """Threads of the oracle's parallel loops (default: every host core);
    returns the count in effect."""
    return int(lib().oracle_set_num_threads(int(nth or host_cores())))


def arpack_eigsh(A, k, **kw):
    """scipy's ARPACK eigsh (the reference's ground truth)."""
    from scipy.sparse.linalg import eigsh

    w, v = eigsh(A, k=k, **kw)
    order = np.argsort(w)
    return w[order], v[:, order]
