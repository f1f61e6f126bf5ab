"""Command line: eigenpairs of a Matrix Market matrix on the GPU.

    python -m gpu_eigsh matrix.mtx [-k 20] [--which SA] [--ncv N] [--tol 1e-10]
                        [--sigma S] [--maxiter N] [--mixed] [--reorder]
                        [--evals out.txt] [--evecs out.npy]

Prints the eigenvalues (ascending), the solve time and the Lanczos step
count; optionally saves them and the eigenvectors (n x k).  The reference's
driver (src/main.cu) builds its own kNN test matrix and compares three
Lanczos variants; this entry point solves the matrix it is given.
"""
from __future__ import annotations

import argparse
import sys
import time

import numpy as np


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m gpu_eigsh", description=__doc__.splitlines()[0])
    ap.add_argument("matrix", help="Matrix Market coordinate file (symmetric matrix)")
    ap.add_argument("-k", type=int, default=20)
    ap.add_argument("--which", default="SA", choices=["LM", "SM", "LA", "SA", "BE"])
    ap.add_argument("--ncv", type=int, default=0)
    ap.add_argument("--tol", type=float, default=1e-10)
    ap.add_argument("--maxiter", type=int, default=None)
    ap.add_argument("--sigma", type=float, default=None)
    ap.add_argument("--mixed", action="store_true", help="fp32 matrix values, fp64 accumulation")
    ap.add_argument("--reorder", action="store_true", help="Cuthill-McKee renumbering inside the solver")
    ap.add_argument("--evals", help="write the eigenvalues to this text file")
    ap.add_argument("--evecs", help="write the eigenvectors (n x k) to this .npy file")
    a = ap.parse_args(argv)

    from . import gpu_eigsh
    from .io import mmread

    t0 = time.perf_counter()
    A = mmread(a.matrix)
    t1 = time.perf_counter()
    if A.shape[0] != A.shape[1]:
        print(f"error: matrix must be square, got {A.shape}", file=sys.stderr)
        return 2
    (w, V), info = gpu_eigsh(A, k=a.k, ncv=a.ncv or None, which=a.which, tol=a.tol, maxiter=a.maxiter,
                             sigma=a.sigma, mixed=a.mixed, reorder=a.reorder, return_info=True,
                             return_eigenvectors=True)
    t2 = time.perf_counter()
    print(f"{a.matrix}: n={A.shape[0]} nnz={A.nnz}  read {t1 - t0:.2f} s  solve {t2 - t1:.2f} s  "
          f"({info['steps']} Lanczos steps, {info['restarts']} restarts)")
    for i, x in enumerate(w):
        print(f"{i:4d}  {x:.15g}")
    if a.evals:
        np.savetxt(a.evals, w, fmt="%.17g")
    if a.evecs:
        np.save(a.evecs, V)
    return 0


if __name__ == "__main__":
    sys.exit(main())
