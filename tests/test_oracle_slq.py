"""CPU: the SLQ / Kraemer / IMGP oracle (oracle/slq.py) reproduces the golden
vectors that the reference's own torch code produced (tests/golden/make_golden.py).

This pins the oracle; the GPU tests then compare the CUDA path with the same
fixtures and with the oracle on further inputs."""
import numpy as np
import pytest
import torch

from oracle import slq as O


def _load(golden_dir, name):
    return np.load(golden_dir / f"{name}.npz")


def test_imgp_matvec_golden(golden_dir):
    d = _load(golden_dir, "imgp_matvec")
    idx = torch.from_numpy(d["idx"])
    d2 = torch.from_numpy(d["d2"])
    kap = torch.tensor(float(d["kappa"]), dtype=torch.float64)
    ell = torch.tensor(float(d["ell"]), dtype=torch.float64)
    diag, triu = O.laplacian_pieces(d2, idx, 200, kap)
    lv = O.lsym_matmul(torch.from_numpy(d["v"]), diag, triu, idx)
    np.testing.assert_allclose(lv.numpy(), d["lsym_v"], rtol=1e-13, atol=1e-13)
    for nu in (1, 2):
        mv = O.make_precision_matvec(d2, idx, 200, nu)
        np.testing.assert_allclose(mv(torch.from_numpy(d["v"]), ell, kap).numpy(), d[f"prec_v_nu{nu}"], rtol=1e-12)
        np.testing.assert_allclose(mv(torch.from_numpy(d["X"]), ell, kap).numpy(), d[f"prec_X_nu{nu}"], rtol=1e-12)


@pytest.mark.parametrize("tag,dtype,tol", [("f64", torch.float64, 1e-10), ("f32", torch.float32, 1e-5)])
def test_slq_imgp_golden(golden_dir, tag, dtype, tol):
    d = _load(golden_dir, f"slq_imgp_{tag}")
    idx = torch.from_numpy(d["idx"])
    d2 = torch.from_numpy(d["d2"]).to(dtype)
    n = int(d["n"])
    for kap, el, nu, mp, lm, seed, ld_ref, ge_ref, gk_ref in d["cases"]:
        mv = O.make_precision_matvec(d2, idx, n, int(nu))
        k_ = torch.tensor(kap, dtype=dtype, requires_grad=True)
        e_ = torch.tensor(el, dtype=dtype, requires_grad=True)
        ld = O.slq_logdet(mv, n, (e_, k_), m_probes=int(mp), lanczos_m=int(lm), seed=int(seed), dtype=dtype)
        ld.backward()
        np.testing.assert_allclose([float(ld), float(e_.grad), float(k_.grad)], [ld_ref, ge_ref, gk_ref],
                                   rtol=tol)


def test_slq_dense_golden(golden_dir):
    d = _load(golden_dir, "slq_dense_f64")
    L = torch.from_numpy(d["L"])
    for c, ld_ref, gc_ref in d["rows"]:
        c_t = torch.tensor(c, dtype=torch.float64, requires_grad=True)
        ld = O.slq_logdet(lambda x, cc: cc * x + L @ x, 50, (c_t,), m_probes=40, lanczos_m=30, seed=123)
        ld.backward()
        np.testing.assert_allclose([float(ld), float(c_t.grad)], [ld_ref, gc_ref], rtol=1e-11)


def test_lanczos_batched_golden(golden_dir):
    d = _load(golden_dir, "lanczos_batched")
    A = torch.from_numpy(d["A"])
    V, al, be, zn = O.lanczos_batched(lambda X: A @ X, torch.from_numpy(d["Z"]), 15)
    np.testing.assert_allclose(al.numpy(), d["alpha"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(be.numpy(), d["betas"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(zn.numpy(), d["znorm"], rtol=1e-14)
    np.testing.assert_allclose(V[:, :, 15].numpy(), d["V_last"], rtol=1e-8, atol=1e-10)


@pytest.mark.parametrize("key", ["20_10_log", "50_30_sqrt", "50_30_inv", "20_10_exp", "100_50_log"])
def test_kraemer_golden(golden_dir, key):
    d = _load(golden_dir, "kraemer_f64")
    n, m, func = key.split("_")
    A = torch.from_numpy(d[f"A_{key}"]).requires_grad_(True)
    v = torch.from_numpy(d[f"v_{key}"]).requires_grad_(True)
    y = O.funm_apply_kraemer(A, v, int(m), func)
    (y * torch.from_numpy(d[f"gy_{key}"])).sum().backward()
    np.testing.assert_allclose(y.detach().numpy(), d[f"y_{key}"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(A.grad.numpy(), d[f"gA_{key}"], rtol=1e-7, atol=1e-9)
    np.testing.assert_allclose(v.grad.numpy(), d[f"gv_{key}"], rtol=1e-7, atol=1e-9)


@pytest.mark.parametrize("key", ["20_10_log", "50_30_inv"])
def test_qform_golden(golden_dir, key):
    d = _load(golden_dir, "qform_op_f64")
    n, m, func = key.split("_")
    A = torch.from_numpy(d[f"A_{key}"]).requires_grad_(True)
    z = torch.from_numpy(d[f"z_{key}"]).requires_grad_(True)
    q = O.funm_qform_op(lambda x, AA: AA @ x, z, (A,), int(m), func)
    q.backward()
    np.testing.assert_allclose(float(q), float(d[f"q_{key}"]), rtol=1e-11)
    np.testing.assert_allclose(z.grad.numpy(), d[f"gz_{key}"], rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(A.grad.numpy(), d[f"gA_{key}"], rtol=1e-8, atol=1e-10)
