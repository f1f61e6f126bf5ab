"""CPU: the schedule of the restart's multishift bulge chase (lg_restart.cu).

The restart applies np exact shifts to the tridiagonal T by chasing one bulge
per shift.  The kernel pipelines up to 32 bulges three rows apart (bulge l of a
batch is at row bs + step - 3 l), computes the rotations of two steps per block
barrier, and applies each pair of steps to Q bulge by bulge.  Emulated here in
numpy with one rotation formula for every schedule, the pipelined and paired
chase must give bitwise the d, e and Q of the plain shift-after-shift chase
(the reference's order, src/tridiag.cuh:67-124 of the reference).
"""
import numpy as np


def _givens(a, b):
    if b == 0.0:
        return 1.0, 0.0
    rh = 1.0 / np.sqrt(a * a + b * b)
    sg = (-1.0 if b > 0.0 else 1.0) if abs(b) > abs(a) else (1.0 if a >= 0.0 else -1.0)
    return sg * a * rh, -sg * b * rh


def _rotate(d, e, k, bs, be, sigma, bulge):
    """One rotation of a bulge at row k (the kernel's arithmetic, in its
    order); returns (c, s, new bulge)."""
    if k == bs:
        c, s = _givens(d[bs] - sigma, e[bs])
    else:
        c, s = _givens(e[k - 1], bulge)
        e[k - 1] = c * e[k - 1] - s * bulge
    dk, dk1, ek = d[k], d[k + 1], e[k]
    cc, ss, cs = c * c, s * s, c * s
    d[k] = cc * dk - 2.0 * cs * ek + ss * dk1
    d[k + 1] = ss * dk + 2.0 * cs * ek + cc * dk1
    e[k] = cs * (dk - dk1) + (cc - ss) * ek
    if k + 1 < be:
        bulge = -s * e[k + 1]
        e[k + 1] = c * e[k + 1]
    return c, s, bulge


def _apply_q(Q, k, c, s):
    x0, x1 = Q[:, k].copy(), Q[:, k + 1].copy()
    Q[:, k] = c * x0 - s * x1
    Q[:, k + 1] = s * x0 + c * x1


def _sequential(d, e, shifts, bs, be):
    d, e, Q = d.copy(), e.copy(), np.eye(len(d))
    for sigma in shifts:
        bulge = 0.0
        for k in range(bs, be):
            c, s, bulge = _rotate(d, e, k, bs, be, sigma, bulge)
            _apply_q(Q, k, c, s)
    return d, e, Q


def _paired_pipeline(d, e, shifts, bs, be, lanes=32):
    d, e, Q = d.copy(), e.copy(), np.eye(len(d))
    for b0 in range(0, len(shifts), lanes):
        nb = min(lanes, len(shifts) - b0)
        steps = (be - bs) + 3 * (nb - 1)
        bulge = [0.0] * nb
        for pr in range((steps + 1) // 2):
            rots = []   # (q, lane, k, c, s) of this pair
            for q in range(2):
                st = 2 * pr + q
                if st >= steps:
                    continue
                # the lanes of one step touch disjoint rows; go through them
                # last lane first to show that their order does not matter
                for lane in reversed(range(nb)):
                    k = bs + st - 3 * lane
                    if bs <= k < be:
                        c, s, bulge[lane] = _rotate(d, e, k, bs, be, shifts[b0 + lane], bulge[lane])
                        rots.append((q, lane, k, c, s))
            # Q: bulge by bulge (any bulge order), each bulge's two steps in order
            for lane in np.random.default_rng(pr).permutation(nb):
                for q in range(2):
                    for (qq, ll, k, c, s) in rots:
                        if qq == q and ll == lane:
                            _apply_q(Q, k, c, s)
    return d, e, Q


def _tridiagonal(m, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(m) + 4.0, np.abs(rng.standard_normal(m)) + 0.1


def test_paired_pipelined_chase_equals_sequential_chase():
    m = 60
    d, e = _tridiagonal(m, 3)
    e[m - 1] = 0.0
    T = np.diag(d) + np.diag(e[: m - 1], 1) + np.diag(e[: m - 1], -1)
    shifts = np.sort(np.linalg.eigvalsh(T))[:40]    # exact shifts, as the restart uses them
    ref = _sequential(d, e, shifts, 0, m - 1)
    got = _paired_pipeline(d, e, shifts, 0, m - 1)
    for a, b in zip(ref, got):
        assert np.array_equal(a, b)


def test_paired_pipelined_chase_on_a_block_and_few_shifts():
    # an unreduced block inside T (rows 5..40) and an odd number of steps
    m = 48
    d, e = _tridiagonal(m, 7)
    shifts = np.linspace(2.0, 5.0, 7)
    ref = _sequential(d, e, shifts, 5, 40)
    got = _paired_pipeline(d, e, shifts, 5, 40)
    for a, b in zip(ref, got):
        assert np.array_equal(a, b)
