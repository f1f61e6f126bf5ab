"""Build the CPU oracle library (test infrastructure only; see irlm_oracle.c).

    python oracle/build_oracle.py

Tries gcc with OpenMP first (all host cores), then without it.  The output,
liboracle_irlm.so, stays next to this file (git-ignored).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "irlm_oracle.c"
LIB = HERE / "liboracle_irlm.so"


def build(force: bool = False) -> Path:
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    base = [cc, "-O3", "-fPIC", "-std=c11", "-shared", "-o", str(LIB), str(SRC), "-lm"]
    gcc_lib = "/usr/lib/gcc/x86_64-linux-gnu/13/"
    variants = [base[:1] + ["-fopenmp"] + base[1:]]
    if Path(gcc_lib).exists():
        variants.append(base[:1] + ["-fopenmp", "-B" + gcc_lib] + base[1:])
    variants.append(base)
    err = ""
    for cmd in variants:
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode == 0:
            return LIB
        err = res.stderr
    raise RuntimeError("oracle build failed:\n" + err)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
