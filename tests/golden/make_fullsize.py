"""Full-size fixtures of configurations 1 and 3 (the sizes the bench times).

    python tests/golden/make_fullsize.py REFERENCE_ROOT [--only cfg1|cfg3]

Configuration 1 (n = 1e6 kNN graph Laplacian: points uniform in [0,1]^2 with
seed 1, k = 10, union-symmetrised, exp(-d^2/2h^2), L = D - W in fp64):
scipy.sparse.linalg.eigsh (ARPACK, the reference's own ground truth,
tests/test_gradient.py:59-81) with k = 20, which = 'LA', ncv = 60,
tol = 1e-10 and v0 = default_rng(0).standard_normal(n), on L and on its
fp32-rounded copy (the matrix the mixed fp32-values / fp64-accumulation mode
multiplies by).  Writes cfg1_knn1e6_arpack.json: both eigenvalue lists, the
Ritz residual norms, and a fingerprint of the matrix (n, nnz, sums of the
indices and values) that the GPU test checks before comparing.

Configuration 3 (n = 1e6, the undirected edges of the same kNN graph with
their squared lengths; IMGP precision operator nu = 2, lengthscale =
graphbandwidth = 1, fp32; 64 Rademacher probes with seed 0; lanczos_m = 30):
the reference's own torch path, python/gpu_eigsh/imgp.py
make_imgp_precision_matvec and python/gpu_eigsh/funm_torch.py slq_logdet
(:730-781), loaded by file path from REFERENCE_ROOT and run on the host, gives
the log-det and its gradients with respect to lengthscale and
graphbandwidth after backward().  The oracle restatement (oracle/slq.py) runs
the same case as a cross-check.  Writes cfg3_slq1e6_reference.json.

Both runs take minutes on a few host cores (the SLQ case holds ~20 GB of
host memory); the outputs are a few hundred bytes each and are committed.
The generators are deterministic (seeded numpy / torch CPU generators).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
SYNTHETIC = ROOT / "lanczos-gpu_b200" / "gpu_eigsh" / "synthetic.py"


def load_synthetic():
    """The seeded generators (numpy / scipy only), loaded by file path so
    that the CUDA library of the package is not mapped."""
    spec = importlib.util.spec_from_file_location("lg_synthetic_fixture", SYNTHETIC)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def fingerprint(L):
    """Order-sensitive checksums of a CSR matrix (cheap to recompute)."""
    ip = L.indptr.astype(np.int64)
    ix = L.indices.astype(np.int64)
    w = np.arange(1, ix.shape[0] + 1, dtype=np.float64)
    return {"n": int(L.shape[0]), "nnz": int(L.nnz), "indptr_sum": int(ip.sum()), "indices_sum": int(ix.sum()),
            "data_sum": float(L.data.sum()), "data_weighted_sum": float((L.data * (w / w[-1])).sum())}


def cfg1(syn):
    from scipy.sparse.linalg import eigsh

    t0 = time.time()
    L, info = syn.knn_laplacian(1_000_000, k=10, seed=1)
    n = L.shape[0]
    v0 = np.random.default_rng(0).standard_normal(n)
    out = {"workload": "eigsh k=20 which=LA ncv=60 tol=1e-10, v0=default_rng(0).standard_normal(n), on the "
                       "n=1e6 kNN graph Laplacian (uniform points in [0,1]^2, seed 1, k=10, union-symmetrised, "
                       "exp(-d^2/2h^2), L = D - W, fp64)",
           "oracle": "scipy.sparse.linalg.eigsh (ARPACK)", "matrix": fingerprint(L), "h": info["h"],
           "anorm1": float(abs(L).sum(axis=1).max())}
    for tag, M in (("fp64", L), ("fp32_rounded", L.astype(np.float32).astype(np.float64))):
        t1 = time.time()
        w, V = eigsh(M, k=20, which="LA", ncv=60, tol=1e-10, v0=v0)
        o = np.argsort(w)
        w, V = w[o], V[:, o]
        res = np.linalg.norm(M @ V - V * w, axis=0)
        out[tag] = {"eigenvalues": [float(x) for x in w], "residuals": [float(x) for x in res],
                    "seconds": round(time.time() - t1, 1)}
        print(f"cfg1 {tag}: {time.time() - t1:.1f} s, max residual {res.max():.3e}", flush=True)
    out["seconds_total"] = round(time.time() - t0, 1)
    (HERE / "cfg1_knn1e6_arpack.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote cfg1_knn1e6_arpack.json", flush=True)


def cfg3(syn, reference_root: Path):
    import torch

    sys.path.insert(0, str(HERE))
    from make_golden import load_reference

    sys.path.insert(0, str(ROOT))
    from oracle import slq as oslq

    torch.set_num_threads(os.cpu_count() or 1)
    n, nu, probes, m, seed = 1_000_000, 2, 64, 30, 0
    idx, d2 = syn.knn_edge_list(n, k=10, seed=1)
    it = torch.from_numpy(idx)
    dt = torch.from_numpy(d2).to(torch.float32)
    out = {"workload": "slq_logdet of the IMGP precision operator (nu=2, lengthscale=graphbandwidth=1) on the "
                       "undirected edges of the n=1e6 kNN graph (uniform points in [0,1]^2, seed 1, k=10), fp32, "
                       "m_probes=64 (seed 0), lanczos_m=30, forward + backward",
           "edges": int(idx.shape[1]), "edge_checksum": int(idx.sum()), "d2_sum": float(d2.sum())}
    ft, imgp = load_reference(reference_root)
    for tag, make, slq in (("reference", imgp.make_imgp_precision_matvec, ft.slq_logdet),
                           ("oracle", None, oslq.slq_logdet)):
        t1 = time.time()
        if make is not None:
            mv = make(x_edge_dists=dt, idx=it, operator_dim=n, nu=nu)
        else:
            mv = oslq.make_precision_matvec(dt, it, n, nu)
        ell = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        kap = torch.tensor(1.0, dtype=torch.float32, requires_grad=True)
        ld = slq(mv, n, (ell, kap), m_probes=probes, lanczos_m=m, seed=seed, dtype=torch.float32)
        ld.backward()
        out[tag] = {"logdet": float(ld), "grad_lengthscale": float(ell.grad), "grad_graphbandwidth": float(kap.grad),
                    "seconds": round(time.time() - t1, 1)}
        print(f"cfg3 {tag}: {out[tag]}", flush=True)
        del mv, ld
    (HERE / "cfg3_slq1e6_reference.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote cfg3_slq1e6_reference.json", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference_root", type=Path, help="root of the reference checkout (python/gpu_eigsh/...)")
    ap.add_argument("--only", choices=["cfg1", "cfg3"])
    a = ap.parse_args()
    syn = load_synthetic()
    if a.only in (None, "cfg1"):
        cfg1(syn)
    if a.only in (None, "cfg3"):
        cfg3(syn, a.reference_root)


if __name__ == "__main__":
    main()
