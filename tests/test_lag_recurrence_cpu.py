"""The lag-step recurrence of the CUDA engine (lg_gs.cu: gs_lag_project /
gs_lag_correct; lg_irlm.cu: Solver::lag_step, finish_lag), restated in numpy
and checked against in-step CGS2 (two classical Gram-Schmidt passes inside
every step, the reference's CGS + DGKS when DGKS fires, src/lanczos_ops.cuh:
113-192): the same basis, alpha and beta to rounding, and the same Lanczos
relation A V = V T + r e^T.

The lag model, entering step j with u = r1 of step j-1 (one pass) and
rho = ||u||:
    z = A u / rho
    s = V^T u,  t = V^T z                     (one stream of V)
    beta_j = sqrt(||u||^2 - ||s||^2);  alpha_{j-1} += s_{j-1}
    v_j = (u - V s) / beta_j
    v_j^T z = (u^T z - s.t) / beta_j
    r1 = (rho / beta_j)(z - V t - (v_j^T z) v_j)   (second stream)
    alpha_j = rho v_j^T z / beta_j - s_{j-1}
and the extension's last residual gets its delayed pass at the end.
"""
import numpy as np
import scipy.sparse as sp


def _cgs2(A, r0, V0, T0, m):
    """In-step CGS2 from a starting residual r0 orthogonal to V0 (k columns)."""
    n = A.shape[0]
    k = V0.shape[1]
    V = np.zeros((n, m))
    V[:, :k] = V0
    al = np.zeros(m)
    be = np.zeros(m + 1)
    al[:k], be[:k + 1] = T0
    r = r0.copy()
    for j in range(k, m):
        rn = np.linalg.norm(r)
        be[j] = rn
        V[:, j] = r / rn
        w = A @ V[:, j]
        h = V[:, :j + 1].T @ w
        r1 = w - V[:, :j + 1] @ h
        s = V[:, :j + 1].T @ r1
        r = r1 - V[:, :j + 1] @ s
        al[j] = h[j] + s[j]
    be[m] = np.linalg.norm(r)
    return V, al, be, r


def _lag(A, r0, V0, T0, m):
    """Lag steps after the first (in-step) step of the extension."""
    n = A.shape[0]
    k = V0.shape[1]
    V = np.zeros((n, m))
    V[:, :k] = V0
    al = np.zeros(m)
    be = np.zeros(m + 1)
    al[:k], be[:k + 1] = T0
    # first step of the extension: in-step passes
    rn = np.linalg.norm(r0)
    be[k] = rn
    V[:, k] = r0 / rn
    w = A @ V[:, k]
    h = V[:, :k + 1].T @ w
    r1 = w - V[:, :k + 1] @ h
    s = V[:, :k + 1].T @ r1
    u = r1 - V[:, :k + 1] @ s
    al[k] = h[k] + s[k]
    for j in range(k + 1, m):
        rho = np.linalg.norm(u)
        z = A @ (u / rho)
        Vj = V[:, :j]
        s = Vj.T @ u
        t = Vj.T @ z
        b2 = u @ u - s @ s
        assert b2 > 0.5 * (u @ u)           # the DGKS test of the lag step
        b = np.sqrt(b2)
        al[j - 1] += s[j - 1]
        be[j] = b
        vjz = (u @ z - s @ t) / b
        al[j] = rho * vjz / b - s[j - 1]
        vj = (u - Vj @ s) / b
        u = (rho / b) * (z - Vj @ t - vjz * vj)
        V[:, j] = vj
    s = V.T @ u                              # finish_lag
    r = u - V @ s
    al[m - 1] += s[m - 1]
    be[m] = np.linalg.norm(r)
    return V, al, be, r


def _relation_err(A, V, al, be, r):
    m = V.shape[1]
    T = np.diag(al) + np.diag(be[1:m], 1) + np.diag(be[1:m], -1)
    E = A @ V - V @ T
    E[:, -1] -= r
    return np.abs(E).max()


def _matrices():
    rng = np.random.default_rng(0)
    n = 400
    # 2-D grid Laplacian, a random sparse SPD matrix, a diagonal with a wide spectrum
    T1 = sp.diags([-np.ones(19), 2 * np.ones(20), -np.ones(19)], [-1, 0, 1])
    I = sp.identity(20)
    yield (sp.kron(I, T1) + sp.kron(T1, I)).tocsr()
    R = sp.random(n, n, density=0.02, random_state=1)
    yield (R @ R.T + sp.identity(n)).tocsr()
    yield sp.diags(np.geomspace(1e-3, 1e3, n)).tocsr()
    del rng


def test_lag_recurrence_matches_cgs2_from_a_fresh_start():
    for A in _matrices():
        n = A.shape[0]
        r0 = np.random.default_rng(3).standard_normal(n)
        V0 = np.zeros((n, 0))
        a = _cgs2(A, r0, V0, (np.zeros(0), np.zeros(1)), 40)
        b = _lag(A, r0, V0, (np.zeros(0), np.zeros(1)), 40)
        scale = abs(A).sum(axis=1).max()
        assert np.abs(a[0].T @ a[0] - np.eye(40)).max() < 1e-13
        assert np.abs(b[0].T @ b[0] - np.eye(40)).max() < 1e-13
        assert np.abs(a[1] - b[1]).max() <= 1e-12 * scale
        assert np.abs(a[2] - b[2]).max() <= 1e-12 * scale
        assert np.abs(a[0] - b[0]).max() < 1e-9
        assert _relation_err(A, *b) <= 1e-12 * scale


def test_lag_recurrence_after_a_restart():
    """An extension that starts from k kept vectors and a residual orthogonal
    to them (the state after an implicit restart): the first step keeps the
    in-step passes and the rest lag, as in Solver::extend."""
    for A in _matrices():
        n = A.shape[0]
        r0 = np.random.default_rng(5).standard_normal(n)
        V, al, be, r = _cgs2(A, r0, np.zeros((n, 0)), (np.zeros(0), np.zeros(1)), 30)
        # keep the first 12 Lanczos vectors with their tridiagonal and residual
        k = 12
        V0 = V[:, :k]
        rk = V[:, k] * be[k]
        a = _cgs2(A, rk, V0, (al[:k], be[:k + 1]), 30)
        b = _lag(A, rk, V0, (al[:k], be[:k + 1]), 30)
        scale = abs(A).sum(axis=1).max()
        assert np.abs(a[1] - b[1]).max() <= 1e-12 * scale
        assert np.abs(a[2] - b[2]).max() <= 1e-12 * scale
        assert _relation_err(A, *b) <= 1e-12 * scale
