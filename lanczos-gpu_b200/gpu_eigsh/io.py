"""Matrix Market files <-> scipy CSR through the library's parallel host
reader and writer (lg_mtx_read / lg_mtx_write).

The reference reads and writes these files in its benchmark driver
(src/main.cu:129-244: one fscanf per entry, insertion sort per row, "%.15e",
exit on errors); here a `coordinate` file (real, integer or pattern; general,
symmetric or skew-symmetric) becomes a CSR with sorted columns and summed
duplicates, and a written file reads back to the same doubles.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _native

__all__ = ["mmread", "mmwrite"]


def mmread(path) -> "scipy.sparse.csr_matrix":  # noqa: F821
    """The matrix of a Matrix Market coordinate file as a float64 CSR."""
    import scipy.sparse as sp

    h = C.c_void_p()
    nr, nc, nnz = C.c_int(0), C.c_int(0), C.c_longlong(0)
    _native.check(_native.lib.lg_mtx_read(os.fsencode(path), C.byref(h), C.byref(nr), C.byref(nc), C.byref(nnz)))
    try:
        rp = np.empty(nr.value + 1, dtype=np.int32)
        ci = np.empty(max(nnz.value, 1), dtype=np.int32)
        va = np.empty(max(nnz.value, 1), dtype=np.float64)
        PI, PD = C.POINTER(C.c_int), C.POINTER(C.c_double)
        _native.check(_native.lib.lg_mtx_copy(h, rp.ctypes.data_as(PI), ci.ctypes.data_as(PI), va.ctypes.data_as(PD)))
    finally:
        _native.lib.lg_mtx_free(h)
    return sp.csr_matrix((va[:nnz.value], ci[:nnz.value], rp), shape=(nr.value, nc.value))


def mmwrite(path, A, symmetric: bool = False) -> None:
    """Write a scipy sparse matrix as `coordinate real general` (or
    `symmetric`: the lower triangle of a square matrix)."""
    import scipy.sparse as sp

    if not sp.issparse(A):
        raise TypeError("A must be a scipy sparse matrix")
    M = sp.csr_matrix(A, dtype=np.float64)
    M.sum_duplicates()
    rp = np.ascontiguousarray(M.indptr, dtype=np.int32)
    ci = np.ascontiguousarray(M.indices, dtype=np.int32)
    va = np.ascontiguousarray(M.data, dtype=np.float64)
    PI, PD = C.POINTER(C.c_int), C.POINTER(C.c_double)
    _native.check(_native.lib.lg_mtx_write(os.fsencode(path), M.shape[0], M.shape[1], rp.ctypes.data_as(PI),
                                           ci.ctypes.data_as(PI), va.ctypes.data_as(PD), int(bool(symmetric))))
