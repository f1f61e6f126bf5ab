"""Build liblanczos_b200.so (sm_100a) in-tree.

    python lanczos-gpu_b200/build.py [--force] [--verbose]

Every CUDA source under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo, then linked into
gpu_eigsh/_lib/liblanczos_b200.so against the static CUDA runtime, so the
library carries no dependency beyond the driver.  Objects go to _build/.
Rebuilds only what changed (any header change rebuilds everything).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
OUT_DIR = PKG / "gpu_eigsh" / "_lib"
LIB = OUT_DIR / "liblanczos_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3", f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    hdr_time = _newest(headers)
    cc = nvcc()
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time)
        if stale:
            flags = NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])
            jobs.append((src, obj, [cc, *flags, "-c", str(src), "-o", str(obj)]))

    def run(job):
        src, obj, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        return src, res

    failed = []
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for src, res in ex.map(run, jobs):
            if res.returncode != 0 or verbose or ptxas_verbose:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                failed.append(src.name)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(failed))

    objs = [BUILD / (s.stem + ".o") for s in sources]
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < _newest(objs):
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl",
               "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas))


if __name__ == "__main__":
    main()
