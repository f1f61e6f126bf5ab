"""ctypes binding of liblanczos_b200.so (the C ABI in include/lanczos_b200.h).

The library is built in-tree by ``python lanczos-gpu_b200/build.py``.  There is
no CPU fallback: if the library is missing or cannot be loaded, importing this
module raises ImportError.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblanczos_b200.so"

LG_OK = 0
LG_NOCONV = 1
LG_ERR_INVALID = -1
LG_ERR_CUDA = -2
LG_ERR_NOMEM = -3
LG_ERR_TIMEOUT = -4
LG_ERR_NUMERIC = -5
LG_ERR_CG_NOCONV = -6

WHICH = {"LM": 0, "SM": 1, "LA": 2, "SA": 3, "BE": 4}
EXCHANGE = {"auto": 0, "allgather": 1, "halo": 2}
TRANSPORT = {"auto": 0, "nccl": 1, "peer": 2}
LG_PLAN_REORDER_BFS = 1
LG_PLAN_CGS2_INLINE = 2
LG_PLAN_REORDER_DEGREE = 4
LG_OP_DEVICE, LG_OP_HOST, LG_OP_STREAM = 0, 1, 2
# callback types of lg_eigsh_plan_create_op (include/lanczos_b200.h)
MATVEC_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)
MATVEC_STREAM_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p)
KNN_METHODS = {"auto": 0, "cells": 1, "brute": 2}


class EigshOpts(C.Structure):
    _fields_ = [
        ("k", C.c_int),
        ("ncv", C.c_int),
        ("maxiter", C.c_int),
        ("max_steps", C.c_longlong),
        ("tol", C.c_double),
        ("which", C.c_int),
        ("use_sigma", C.c_int),
        ("sigma", C.c_double),
        ("cg_max_iters", C.c_int),
        ("cg_tol", C.c_double),
        ("mixed", C.c_int),
        ("seed", C.c_uint64),
        ("return_vectors", C.c_int),
        ("evecs_rowmajor", C.c_int),
        ("profile", C.c_int),
    ]


KERNEL_CLASSES = ["spmv", "gs_project", "gs_correct_project", "gs_correct", "restart", "basis", "cg", "other", "comm"]


class EigshInfo(C.Structure):
    _fields_ = [
        ("nconv", C.c_int),
        ("restarts", C.c_int),
        ("steps", C.c_longlong),
        ("pass3", C.c_int),
        ("breakdowns", C.c_int),
        ("cg_iters", C.c_longlong),
        ("cg_failures", C.c_int),
        ("ms", C.c_double),
        ("launches", C.c_longlong),
        ("kernel_ms", C.c_double * len(KERNEL_CLASSES)),
        ("kernel_calls", C.c_longlong * len(KERNEL_CLASSES)),
        ("kernel_bytes", C.c_double * len(KERNEL_CLASSES)),
    ]

    def as_dict(self) -> dict:
        out = {}
        for name, _ in self._fields_:
            v = getattr(self, name)
            if name.startswith("kernel_"):
                v = {cls: v[i] for i, cls in enumerate(KERNEL_CLASSES)}
            out[name] = v
        return out


LG_F32 = 0
LG_F64 = 1
FUNCS = {"log": 0, "exp": 1, "sqrt": 2, "inv": 3}


class SlqOp(C.Structure):
    """lg_slq_op: P = (shift I + L)^power, L = diag + off-diagonal CSR."""
    _fields_ = [
        ("n", C.c_int),
        ("nnz", C.c_longlong),
        ("rowptr", C.c_void_p),
        ("col", C.c_void_p),
        ("offval", C.c_void_p),
        ("diag", C.c_void_p),
        ("doffval", C.c_void_p),
        ("ddiag", C.c_void_p),
        ("shift", C.c_double),
        ("power", C.c_int),
        ("dtype", C.c_int),
    ]


_PD = C.POINTER(C.c_double)
_PI = C.POINTER(C.c_int)
_V = C.c_void_p
_I = C.c_int
_SZ = C.c_size_t
_POP = C.POINTER(SlqOp)

# Every exported symbol with its ctypes signature (restype, argtypes).
SIGNATURES = {
    "lg_eigsh_opts_default": (C.c_int, [C.POINTER(EigshOpts)]),
    "lg_eigsh_plan_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_longlong, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "lg_eigsh_plan_create_ex": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_longlong, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]),
    "lg_eigsh_plan_create_op": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_int]),
    "lg_eigsh_plan_run": (C.c_int, [C.c_void_p, C.POINTER(EigshOpts), C.c_void_p, _PD, C.c_void_p, C.c_int,
                                    C.POINTER(EigshInfo)]),
    "lg_eigsh_plan_destroy": (C.c_int, [C.c_void_p]),
    "lg_comm_unique_id": (C.c_int, [C.c_void_p, C.c_int]),
    "lg_comm_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "lg_comm_destroy": (C.c_int, [C.c_void_p]),
    "lg_partition_block": (C.c_int, [C.c_int, C.c_int]),
    "lg_eigsh_plan_create_dist": (C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_int, C.c_int, C.c_longlong,
                                            C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "lg_eigsh_plan_set_exchange": (C.c_int, [C.c_void_p, C.c_int]),
    "lg_eigsh_plan_set_transport": (C.c_int, [C.c_void_p, C.c_int]),
    "lg_eigsh_plan_transport": (C.c_int, [C.c_void_p, _PI]),
    "lg_halo_recv_list": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_longlong, _PI, _PI, C.c_longlong,
                                    C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
    "lg_halo_send_plan": (C.c_int, [C.c_int, C.c_int, C.c_int, _PD, C.POINTER(C.c_longlong), _PI]),
    "lg_eigsh_plan_exchange_info": (C.c_int, [C.c_void_p, _PI, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
    "lg_eigsh_plan_matvec": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "lg_eigsh_plan_factorize": (C.c_int, [C.c_void_p, _PD, C.c_int, _PD, _PD]),
    "lg_eigsh": (C.c_int, [C.c_int, C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(EigshOpts),
                           C.c_void_p, _PD, C.c_void_p, C.POINTER(EigshInfo)]),
    "lg_cgs2_orthogonalize": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p]),
    "lg_cgs2_orthogonalize_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "lg_slq_workspace_bytes": (_SZ, [_POP, _I, _I]),
    "lg_slq_forward": (_I, [_POP, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_backward": (_I, [_POP, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_apply": (_I, [_POP, _I, _I, _V, _V, _V, _SZ, _V]),
    "lg_slq_apply_vjp": (_I, [_POP, _I, _I, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_small_side": (_I, [_I, _I, _I, _I, _V, _V, _V, _V, C.c_double, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_block_start": (_I, [_I, _I, _I, _I, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_block_step": (_I, [_I, _I, _I, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_block_lambda": (_I, [_I, _I, _I, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_block_xi": (_I, [_I, _I, _I, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_slq_block_start_grad": (_I, [_I, _I, _I, _I, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "lg_imgp_laplacian": (_I, [_I, C.c_longlong, _V, _V, _I, _V, C.c_double, _I, _V, _V, _V, _V, _V, _V]),
    "lg_graph_bfs_levels": (_I, [_I, _V, _V, _I, _V, _V, _PI, _V]),
    "lg_graph_cm_order": (_I, [_I, _PI, _PI, _PI]),
    "lg_mtx_read": (_I, [C.c_char_p, C.POINTER(C.c_void_p), _PI, _PI, C.POINTER(C.c_longlong)]),
    "lg_mtx_copy": (_I, [_V, _PI, _PI, _PD]),
    "lg_mtx_free": (_I, [_V]),
    "lg_mtx_write": (_I, [C.c_char_p, _I, _I, _PI, _PI, _PD, _I]),
    "lg_knn": (_I, [_I, _I, _I, _V, _V, _V, _I, _V]),
    "lg_knn_laplacian_rows": (_I, [_I, _I, _V, _V, C.POINTER(C.c_longlong), _V]),
    "lg_knn_laplacian_fill": (_I, [_I, _I, _V, _V, C.c_double, _V, _V, _V, _V]),
    "lg_dense_matvec": (_I, [_I, _I, _V, _V, _I, _V, _I, _V]),
    "lg_outer_accumulate": (_I, [_I, _I, _V, _V, _I, _V, _V]),
    "lg_eigsh_adjoint": (_I, [_I, C.c_longlong, _V, _V, _V, _I, _V, _V, _V, _V, _V, _I, C.c_double, _PI, _V]),
    "compute_adjoint_eigsh": (_I, [_I, _I, _PI, _PI, _PD, _I, _PD, _PD, _PD, _PD, _PD, _I, C.c_double]),
    "lg_eigsh_plan_funm": (_I, [_V, _V, _I, _I, _I, _I, _V, _PD, _PI]),
    "compute_funm_apply": (_I, [_I, _I, _PI, _PI, _PD, _PD, _I, C.c_char_p, _PD]),
    "compute_funm_qform": (_I, [_I, _I, _PI, _PI, _PD, _PD, _I, C.c_char_p, _PD]),
    "compute_funm_debug": (_I, [_I, _I, _PI, _PI, _PD, _PD, _I, _PD, _PD, _PD]),
    "lg_status_string": (C.c_char_p, [C.c_int]),
    "lg_last_error": (C.c_int, [C.c_char_p, C.c_int]),
    "compute_eigsh": (C.c_int, [C.c_int, C.c_int, _PI, _PI, _PD, C.c_int, C.c_int, C.c_int, C.c_double, _PD,
                                _PD]),
    "compute_eigsh_sigma": (C.c_int, [C.c_int, C.c_int, _PI, _PI, _PD, C.c_int, C.c_int, C.c_int, C.c_double,
                                      C.c_double, C.c_int, C.c_double, _PD, _PD]),
}


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"{_LIB_PATH} is missing; build it with `python lanczos-gpu_b200/build.py` "
            "(nvcc, sm_100a).  There is no CPU fallback.")
    lib = C.CDLL(str(_LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
LIB_PATH = str(_LIB_PATH)


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib.lg_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def status_string(rc: int) -> str:
    return lib.lg_status_string(rc).decode()


class LanczosError(RuntimeError):
    """A failure reported by the CUDA engine (status code + message)."""

    def __init__(self, rc: int, msg: str = ""):
        self.status = rc
        super().__init__(f"{status_string(rc)} ({rc}): {msg or last_error()}")


def check(rc: int) -> int:
    if rc < 0:
        raise LanczosError(rc)
    return rc


def ptr(a) -> int:
    """Address of a C-contiguous numpy array (or 0 for None)."""
    if a is None:
        return 0
    return a.ctypes.data
