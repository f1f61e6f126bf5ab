"""Generate golden vectors for the SLQ / Kraemer / IMGP path from the reference's
own torch code.

    python tests/golden/make_golden.py REFERENCE_ROOT

REFERENCE_ROOT is the root of a checkout of the reference.  The reference modules
python/gpu_eigsh/funm_torch.py and imgp.py are loaded by file path (the
package __init__ would import the CUDA extension, which is not built here).
Outputs small .npz files next to this script; they are committed, and the
tests read them without the reference present.

Cases (all seeded; inputs are stored with the outputs):
  imgp_matvec.npz        L_sym(kappa) v and P(theta, kappa) v (nu = 1, 2), fp64
  slq_imgp_f64.npz       slq_logdet on the IMGP precision operator, fp64:
                         log det and d/d lengthscale, d/d graphbandwidth
  slq_imgp_f32.npz       the same in fp32
  slq_dense_f64.npz      slq_logdet of A(c) = c I + L (dense L), d/dc
  lanczos_batched.npz    alpha / beta of the batched no-reortho recurrence
  kraemer_f64.npz        funm_apply_kraemer y, grad_A, grad_v (log/sqrt/inv/exp)
  qform_op_f64.npz       funm_qform_op q, grad_z, grad_A
"""
from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    pkgdir = root / "python" / "gpu_eigsh"
    pkg = types.ModuleType("gpu_eigsh_ref")
    pkg.__path__ = [str(pkgdir)]
    sys.modules["gpu_eigsh_ref"] = pkg
    mods = {}
    for name in ("funm_torch", "imgp"):
        spec = importlib.util.spec_from_file_location(f"gpu_eigsh_ref.{name}", pkgdir / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"gpu_eigsh_ref.{name}"] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["funm_torch"], mods["imgp"]


def knn_edges(n, dim=5, k=10, seed=0):
    """Edge list in the IMGP format (src < dst kept from the directed kNN list),
    the construction of the reference's tests/test_imgp_integration.py:33-59."""
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((n, dim))
    d, ix = cKDTree(pts).query(pts, k=k + 1)
    src = np.repeat(np.arange(n), k)
    dst = ix[:, 1:].ravel()
    d2 = (d[:, 1:] ** 2).ravel()
    keep = src < dst
    return np.stack([src[keep], dst[keep]]).astype(np.int64), d2[keep]


def spd(n, seed):
    g = torch.Generator().manual_seed(seed)
    M = torch.randn(n, n, generator=g, dtype=torch.float64)
    return M @ M.T + n * torch.eye(n, dtype=torch.float64)


def main(root: Path):
    ft, imgp = load_reference(root)
    out = {}

    # ---- IMGP matvecs ------------------------------------------------------
    idx, d2 = knn_edges(200, seed=0)
    rng = np.random.default_rng(1)
    v = rng.standard_normal(200)
    X = rng.standard_normal((200, 8))
    it, dt = torch.from_numpy(idx), torch.from_numpy(d2)
    kappa = torch.tensor(1.3, dtype=torch.float64)
    ell = torch.tensor(0.7, dtype=torch.float64)
    lv = imgp._matmul_symmetric_laplacian(torch.from_numpy(v), dt, it, 200, kappa, True)
    res = {"idx": idx, "d2": d2, "v": v, "X": X, "kappa": 1.3, "ell": 0.7, "lsym_v": lv.numpy()}
    for nu in (1, 2):
        mv = imgp.make_imgp_precision_matvec(x_edge_dists=dt, idx=it, operator_dim=200, nu=nu)
        res[f"prec_v_nu{nu}"] = mv(torch.from_numpy(v), ell, kappa).numpy()
        res[f"prec_X_nu{nu}"] = mv(torch.from_numpy(X), ell, kappa).numpy()
    out["imgp_matvec"] = res

    # ---- SLQ on the IMGP operator ------------------------------------------
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        n = 300
        idx, d2 = knn_edges(n, seed=3)
        it, dt = torch.from_numpy(idx), torch.from_numpy(d2).to(dtype)
        cases = []
        for (kap, el, nu, mp, lm, seed) in ((1.0, 1.0, 2, 16, 20, 0), (2.0, 0.5, 2, 32, 30, 5),
                                            (0.7, 1.5, 1, 8, 25, 11)):
            mv = imgp.make_imgp_precision_matvec(x_edge_dists=dt, idx=it, operator_dim=n, nu=nu)
            k_ = torch.tensor(kap, dtype=dtype, requires_grad=True)
            e_ = torch.tensor(el, dtype=dtype, requires_grad=True)
            ld = ft.slq_logdet(mv, n, (e_, k_), m_probes=mp, lanczos_m=lm, seed=seed, dtype=dtype, device="cpu")
            ld.backward()
            cases.append([kap, el, nu, mp, lm, seed, float(ld), float(e_.grad), float(k_.grad)])
        out[f"slq_imgp_{tag}"] = {"idx": idx, "d2": d2, "n": n, "cases": np.array(cases, dtype=np.float64)}

    # ---- SLQ on A(c) = c I + L (dense) ------------------------------------
    n = 50
    L = spd(n, 7)
    rows = []
    for c in (1.0, 5.0, 10.0):
        c_t = torch.tensor(c, dtype=torch.float64, requires_grad=True)
        ld = ft.slq_logdet(lambda x, cc: cc * x + L @ x, n, (c_t,), m_probes=40, lanczos_m=30, seed=123,
                           dtype=torch.float64, device="cpu")
        ld.backward()
        rows.append([c, float(ld), float(c_t.grad)])
    out["slq_dense_f64"] = {"L": L.numpy(), "rows": np.array(rows)}

    # ---- batched recurrence --------------------------------------------------
    n, B, m = 120, 6, 15
    A = spd(n, 21) / n
    g = torch.Generator().manual_seed(3)
    Z = torch.randint(0, 2, (n, B), generator=g, dtype=torch.float64) * 2 - 1
    V, al, be, zn = ft.lanczos_torch_noreortho_batched(lambda X: A @ X, Z, m)
    out["lanczos_batched"] = {"A": A.numpy(), "Z": Z.numpy(), "alpha": al.numpy(), "betas": be.numpy(),
                              "znorm": zn.numpy(), "V_last": V[:, :, m].numpy()}

    # ---- Kraemer adjoint (dense A) -------------------------------------------
    res = {}
    for (n, m, func) in ((20, 10, "log"), (50, 30, "sqrt"), (50, 30, "inv"), (20, 10, "exp"), (100, 50, "log")):
        A = spd(n, n)
        g = torch.Generator().manual_seed(n + 1)
        v = torch.randn(n, generator=g, dtype=torch.float64)
        gy = torch.randn(n, generator=g, dtype=torch.float64)
        A1 = A.clone().requires_grad_(True)
        v1 = v.clone().requires_grad_(True)
        y = ft.funm_apply_kraemer(A1, v1, m, func)
        (y * gy).sum().backward()
        key = f"{n}_{m}_{func}"
        res[f"A_{key}"] = A.numpy()
        res[f"v_{key}"] = v.numpy()
        res[f"gy_{key}"] = gy.numpy()
        res[f"y_{key}"] = y.detach().numpy()
        res[f"gA_{key}"] = A1.grad.numpy()
        res[f"gv_{key}"] = v1.grad.numpy()
    out["kraemer_f64"] = res

    # ---- operator-callable quadratic form -------------------------------------
    res = {}
    for (n, m, func) in ((20, 10, "log"), (50, 30, "inv")):
        A = spd(n, n)
        g = torch.Generator().manual_seed(n + 1)
        z = torch.randn(n, generator=g, dtype=torch.float64)
        A1 = A.clone().requires_grad_(True)
        z1 = z.clone().requires_grad_(True)
        q = ft.funm_qform_op(lambda x, Ap: Ap @ x, z1, (A1,), m, func)
        q.backward()
        key = f"{n}_{m}_{func}"
        res[f"A_{key}"] = A.numpy()
        res[f"z_{key}"] = z.numpy()
        res[f"q_{key}"] = np.array(float(q))
        res[f"gz_{key}"] = z1.grad.numpy()
        res[f"gA_{key}"] = A1.grad.numpy()
    out["qform_op_f64"] = res

    for name, d in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **d)
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_ROOT")
    main(Path(sys.argv[1]))
