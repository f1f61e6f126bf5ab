"""GPU parity at the sizes the bench times (configurations 1 and 3).

Fixtures (tests/golden/make_fullsize.py, committed):
  cfg1_knn1e6_arpack.json   scipy ARPACK eigsh (k=20, LA, ncv=60, tol=1e-10,
                            v0 = default_rng(0)) on the n = 1e6 kNN Laplacian
                            and on its fp32-rounded copy;
  cfg3_slq1e6_reference.json  the reference's own torch slq_logdet + backward
                            (python/gpu_eigsh/funm_torch.py:730-781 on the
                            operator of python/gpu_eigsh/imgp.py:234-289) on
                            the same graph's edges, fp32, 64 probes (seed 0),
                            lanczos_m = 30.

Bars: eigenvalues within 1e-10 relative of ARPACK in fp64 and in the mixed
mode against ARPACK on the fp32-rounded matrix (every eigenvalue here is
about 17, none is near zero), every residual <= tol * ||A||; log-det and both
gradients within 1e-5 relative of the reference in fp32.
"""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg1(golden_dir):
    from gpu_eigsh import synthetic as syn

    fx = json.loads((golden_dir / "cfg1_knn1e6_arpack.json").read_text())
    L, _ = syn.knn_laplacian(1_000_000, k=10, seed=1)
    fp = fx["matrix"]
    # the generator rebuilt the fixture's matrix (exact structure, values to rounding)
    assert (L.shape[0], L.nnz) == (fp["n"], fp["nnz"])
    assert int(L.indptr.astype(np.int64).sum()) == fp["indptr_sum"]
    assert int(L.indices.astype(np.int64).sum()) == fp["indices_sum"]
    w = np.arange(1, L.nnz + 1, dtype=np.float64)
    assert abs(float((L.data * (w / w[-1])).sum()) - fp["data_weighted_sum"]) < 1e-9
    v0 = np.random.default_rng(0).standard_normal(L.shape[0])
    return L, v0, fx


@pytest.mark.parametrize("mode", ["fp64", "mixed"])
def test_cfg1_eigenvalues_equal_arpack(cfg1, mode):
    import torch

    import gpu_eigsh

    L, v0, fx = cfg1
    ref = np.array(fx["fp64" if mode == "fp64" else "fp32_rounded"]["eigenvalues"])
    n = L.shape[0]
    dev = torch.device("cuda")
    rp = torch.from_numpy(L.indptr.astype(np.int32)).to(dev)
    ci = torch.from_numpy(L.indices.astype(np.int32)).to(dev)
    va = torch.from_numpy(L.data).to(dev)
    v0d = torch.from_numpy(v0).to(dev)
    Y = torch.empty((n, 20), dtype=torch.float64, device=dev)
    # the bench's plan: Cuthill-McKee renumbering inside, device buffers
    with gpu_eigsh.EigshPlan(None, max_ncv=60, mixed=(mode == "mixed"), reorder=True,
                             device_csr=(n, L.nnz, rp.data_ptr(), ci.data_ptr(), va.data_ptr())) as plan:
        w, _ = plan.solve(k=20, which="LA", ncv=60, tol=1e-10, v0_device=v0d.data_ptr(), evecs_out=Y.data_ptr())
        info = dict(plan.last_info)
    assert info["nconv"] >= 20
    rel = np.abs(w - ref) / np.abs(ref)
    assert rel.max() < 1e-10, (mode, rel.max(), w, ref)
    # residuals against the matrix the mode multiplies by, in the caller's numbering
    M = L if mode == "fp64" else L.astype(np.float32).astype(np.float64)
    V = Y.cpu().numpy()
    res = np.linalg.norm(M @ V - V * w, axis=0)
    assert res.max() <= 1e-10 * fx["anorm1"]
    assert np.abs(V.T @ V - np.eye(20)).max() < 1e-9


def test_cfg3_slq_equals_reference_fp32(golden_dir):
    import torch

    from gpu_eigsh import synthetic as syn
    from gpu_eigsh.funm_torch import slq_logdet
    from gpu_eigsh.imgp import make_imgp_precision_matvec

    fx = json.loads((golden_dir / "cfg3_slq1e6_reference.json").read_text())
    n = 1_000_000
    idx, d2 = syn.knn_edge_list(n, k=10, seed=1)
    assert int(idx.shape[1]) == fx["edges"] and int(idx.sum()) == fx["edge_checksum"]
    dev = torch.device("cuda")
    mv = make_imgp_precision_matvec(x_edge_dists=torch.from_numpy(d2).to(dev, torch.float32),
                                    idx=torch.from_numpy(idx).to(dev), operator_dim=n, nu=2)
    ell = torch.tensor(1.0, dtype=torch.float32, device=dev, requires_grad=True)
    kap = torch.tensor(1.0, dtype=torch.float32, device=dev, requires_grad=True)
    ld = slq_logdet(mv, n, (ell, kap), m_probes=64, lanczos_m=30, seed=0, dtype=torch.float32, device=dev)
    ld.backward()
    ref = fx["reference"]
    got = {"logdet": float(ld.detach()), "grad_lengthscale": float(ell.grad), "grad_graphbandwidth": float(kap.grad)}
    for key, val in got.items():
        assert abs(val - ref[key]) <= 1e-5 * abs(ref[key]), (key, val, ref[key])
