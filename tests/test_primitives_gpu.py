"""GPU: the CGS2 re-orthogonalisation primitive against a torch fp64 reference."""
import pytest

pytestmark = pytest.mark.gpu


def _basis(n, ldv, ncols, seed, torch):
    g = torch.Generator(device="cuda").manual_seed(seed)
    Q, _ = torch.linalg.qr(torch.randn(n, ncols, generator=g, device="cuda", dtype=torch.float64))
    V = torch.full((n, ldv), float("nan"), device="cuda", dtype=torch.float64)   # padding must never leak in
    V[:, :ncols] = Q
    return V, Q


@pytest.mark.parametrize("n,ncols", [(1000, 3), (50000, 16), (50000, 17), (120000, 31), (120000, 61),
                                     (200000, 64), (100000, 97), (70000, 128)])
def test_cgs2_matches_torch(n, ncols):
    import torch
    from gpu_eigsh.primitives import cgs2_orthogonalize

    ldv = ncols + 2 if ncols % 2 == 0 else ncols + 1
    V, Q = _basis(n, ldv, ncols, 7 + ncols, torch)
    g = torch.Generator(device="cuda").manual_seed(1)
    w = torch.randn(n, generator=g, device="cuda", dtype=torch.float64)
    w = w + 3.0 * (Q @ torch.randn(ncols, generator=g, device="cuda", dtype=torch.float64))
    r, coef, norms = cgs2_orthogonalize(V, ncols, w)
    torch.cuda.synchronize()
    h1 = Q.T @ w
    r1 = w - Q @ h1
    s = Q.T @ r1
    r2 = r1 - Q @ s
    scale = w.norm()
    assert (r - r2).norm() / scale < 1e-12
    assert (coef - (h1 + s)).norm() / (h1 + s).norm() < 1e-12
    ref = torch.stack([w.norm(), r1.norm(), r2.norm()])
    assert ((norms - ref).abs() / ref).max() < 1e-12
    # r is orthogonal to the basis to working precision
    assert (Q.T @ r).abs().max() / scale < 1e-13


def test_cgs2_argument_errors():
    import torch
    from gpu_eigsh import LanczosError
    from gpu_eigsh.primitives import cgs2_orthogonalize

    V = torch.zeros(100, 8, device="cuda", dtype=torch.float64)
    w = torch.ones(100, device="cuda", dtype=torch.float64)
    with pytest.raises(LanczosError):
        cgs2_orthogonalize(V, 9, w)            # ldv too small for ncols
    with pytest.raises(LanczosError):
        cgs2_orthogonalize(V, 4, w, r=w)       # r aliases w
