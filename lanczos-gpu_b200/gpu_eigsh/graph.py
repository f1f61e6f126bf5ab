"""kNN graphs and their Laplacians built on the GPU (lg_knn,
lg_knn_laplacian_rows / lg_knn_laplacian_fill).

The reference builds its test matrices on the host: the driver's brute-force
kNN graph (src/main.cu:30-124, weights exp(-d^2 / (4 bw^2)), union
symmetrisation, L = D - A) and the large-matrix generator
(benchmark/generate_large_laplacian.py: cKDTree on RandomState(seed).random
points, the same weights, A.maximum(A.T), L = D - A, written as Matrix
Market).  Here both run on the device:

  knn(points, k)                        exact neighbours, ascending (d^2, index)
  knn_laplacian(points, k, bw)          L = D - A as a device CSR
  generate_knn_laplacian(n, dim, k, bw, seed)
                                        the generator's matrix, as scipy CSR

and ``python -m gpu_eigsh.graph --n N --dim D --k K --bw BW --seed S --outdir
DIR`` writes DIR/laplacian.mtx like the generator script.
"""
from __future__ import annotations

import argparse
import ctypes as C
import os
import time

import numpy as np
import torch

from . import _native

__all__ = ["knn", "knn_laplacian", "generate_points", "generate_knn_laplacian"]


def _stream(dev):
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _device_points(points) -> torch.Tensor:
    if not torch.is_tensor(points):
        points = torch.from_numpy(np.ascontiguousarray(points, dtype=np.float64))
    if points.dim() != 2:
        raise ValueError(f"points must be (n, dim), got shape {tuple(points.shape)}")
    dev = points.device if points.is_cuda else torch.device("cuda", torch.cuda.current_device())
    return points.to(dev, torch.float64).contiguous()


def knn(points, k: int, method: str = "auto"):
    """Exact k nearest neighbours (self excluded) of the rows of `points`
    ((n, dim), host array or tensor; computed on the GPU).  Returns device
    tensors (idx (n, k) int64, d2 (n, k) float64), each row ascending by
    (squared distance, index).  method: "auto" (cell grid for dim <= 3,
    else all pairs), "cells" or "brute"."""
    if method not in _native.KNN_METHODS:
        raise ValueError(f"method must be one of {sorted(_native.KNN_METHODS)}")
    P = _device_points(points)
    n, dim = P.shape
    k = int(k)
    if not 1 <= k < n:
        raise ValueError(f"k must be in [1, n - 1], got k={k}, n={n}")
    idx = torch.empty((n, k), dtype=torch.int64, device=P.device)
    d2 = torch.empty((n, k), dtype=torch.float64, device=P.device)
    _native.check(_native.lib.lg_knn(n, dim, k, P.data_ptr(), idx.data_ptr(), d2.data_ptr(),
                                     _native.KNN_METHODS[method], _stream(P.device)))
    return idx, d2


def laplacian_from_knn(idx: torch.Tensor, d2: torch.Tensor, bw: float):
    """L = D - A of the union-symmetrised kNN graph with weights
    exp(-d2 / (4 bw^2)), from device neighbour lists.  Returns device
    (rowptr int32 (n+1), col int32 (nnz), val float64 (nnz)), columns
    ascending in every row, diagonal included."""
    if not (bw > 0):
        raise ValueError("bw must be positive")
    n, k = idx.shape
    dev = idx.device
    idx = idx.to(torch.int64).contiguous()
    d2 = d2.to(dev, torch.float64).contiguous()
    rowptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
    nnz = C.c_longlong(0)
    st = _stream(dev)
    _native.check(_native.lib.lg_knn_laplacian_rows(n, k, idx.data_ptr(), rowptr.data_ptr(), C.byref(nnz), st))
    col = torch.empty(nnz.value, dtype=torch.int32, device=dev)
    val = torch.empty(nnz.value, dtype=torch.float64, device=dev)
    _native.check(_native.lib.lg_knn_laplacian_fill(n, k, idx.data_ptr(), d2.data_ptr(), 4.0 * bw * bw,
                                                    rowptr.data_ptr(), col.data_ptr(), val.data_ptr(), st))
    return rowptr, col, val


def knn_laplacian(points, k: int, bw: float, method: str = "auto"):
    """The kNN graph Laplacian of the reference's builders, on the GPU:
    device (rowptr, col, val); see laplacian_from_knn."""
    idx, d2 = knn(points, k, method)
    return laplacian_from_knn(idx, d2, bw)


def generate_points(n: int, dim: int, seed: int) -> np.ndarray:
    """The generator's point cloud: RandomState(seed).random((n, dim))
    (benchmark/generate_large_laplacian.py:29-30)."""
    return np.random.RandomState(seed).random((n, dim))


def generate_knn_laplacian(n: int = 100000, dim: int = 10, k: int = 15, bw: float = 0.3, seed: int = 123,
                           method: str = "auto"):
    """The matrix of benchmark/generate_large_laplacian.py (same defaults),
    built on the GPU.  Returns a scipy CSR (float64)."""
    import scipy.sparse as sp

    rp, col, val = knn_laplacian(generate_points(n, dim, seed), k, bw, method)
    return sp.csr_matrix((val.cpu().numpy(), col.cpu().numpy(), rp.cpu().numpy()), shape=(n, n))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m gpu_eigsh.graph",
                                 description="Generate a kNN graph Laplacian (Matrix Market) on the GPU.")
    ap.add_argument("--n", type=int, default=100000)
    ap.add_argument("--dim", type=int, default=10)
    ap.add_argument("--k", type=int, default=15)
    ap.add_argument("--bw", type=float, default=0.3)
    ap.add_argument("--seed", type=int, default=123)
    ap.add_argument("--method", default="auto", choices=sorted(_native.KNN_METHODS))
    ap.add_argument("--outdir", default="data")
    a = ap.parse_args(argv)
    from .io import mmwrite

    t0 = time.perf_counter()
    L = generate_knn_laplacian(a.n, a.dim, a.k, a.bw, a.seed, a.method)
    t1 = time.perf_counter()
    os.makedirs(a.outdir, exist_ok=True)
    out = os.path.join(a.outdir, "laplacian.mtx")
    mmwrite(out, L)
    t2 = time.perf_counter()
    print(f"Done: n={a.n:,}, nnz={L.nnz:,}, build={t1 - t0:.1f}s, write={t2 - t1:.1f}s")
    print(f"Saved: {out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
