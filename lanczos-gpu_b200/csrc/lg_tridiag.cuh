// lg_tridiag.cuh — small symmetric tridiagonal eigen-kernels shared by the
// IRLM restart (lg_restart.cu) and the SLQ quadrature (lg_slq.cu).
//
//   givens            — plane rotation [c -s; s c][a; b] = [r; 0]
//   sturm_count       — number of eigenvalues below x (LDL^T pivots)
//   inverse_iteration — eigenvector for an accurate eigenvalue by inverse
//                       iteration with a pivoted tridiagonal LU and
//                       re-orthogonalisation against a cluster (the method of
//                       LAPACK dstein), one thread per eigenvalue.
#pragma once

#include "lg_common.cuh"

namespace lg {

constexpr double kUnitRoundoff = 1.1102230246251565e-16;   // 2^-53

// [c -s; s c] [a; b] = [r; 0]; same signs as the classical formulation
// (tau = -a/b or -b/a, Golub & Van Loan 5.1.3) with one reciprocal sqrt.
__device__ __forceinline__ void givens(double a, double b, double& c, double& s) {
  if (b == 0.0) {
    c = 1.0;
    s = 0.0;
    return;
  }
  const double r2 = a * a + b * b;
  const double rh = (r2 >= kSafeMin && r2 < 1e300) ? rsqrt(r2) : 1.0 / hypot(a, b);
  const double sg = (fabs(b) > fabs(a)) ? (b > 0.0 ? -1.0 : 1.0) : (a >= 0.0 ? 1.0 : -1.0);
  c = sg * a * rh;
  s = -sg * b * rh;
}

// 1 / q for |q| >= DBL_MIN: the hardware's approximate reciprocal, refined by
// two Newton-Raphson steps r <- r + r (1 - q r) (each roughly doubles the
// correct bits), to within a couple of units in the last place.  The Sturm
// counts below only need the signs of the pivots; an fp64 division is a long
// instruction sequence, and these counts are the restart's inner loop.
__device__ __forceinline__ double recip_nr(double q) {
  double r;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(q));
  double e = fma(-q, r, 1.0);
  r = fma(r, e, r);
  e = fma(-q, r, 1.0);
  return fma(r, e, r);
}

// Number of eigenvalues of T below x (Sturm sequence of the LDL^T pivots).
__device__ inline int sturm_count(const double* d, const double* e2, int m, double x, double pivmin) {
  double q = d[0] - x;
  int cnt = q < 0.0;
  for (int k = 1; k < m; ++k) {
    if (fabs(q) < pivmin) q = -pivmin;
    q = (d[k] - x) - e2[k - 1] / q;
    cnt += q < 0.0;
  }
  return cnt;
}

// Sturm counts at P points at once: P independent LDL^T pivot chains
// interleaved, so their reciprocals overlap.  Same recurrence as sturm_count,
// with e2 / q formed as e2 * recip_nr(q).
constexpr int kSturmP = 4;
template <int P>
__device__ __forceinline__ void sturm_counts(const double* d, const double* e2, int m, const double* x,
                                             double pivmin, int* cnt) {
  double q[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    q[p] = d[0] - x[p];
    cnt[p] = q[p] < 0.0;
  }
  for (int k = 1; k < m; ++k) {
    const double dk = d[k], ek = e2[k - 1];
#pragma unroll
    for (int p = 0; p < P; ++p) {
      if (fabs(q[p]) < pivmin) q[p] = -pivmin;
      q[p] = (dk - x[p]) - ek * recip_nr(q[p]);
      cnt[p] += q[p] < 0.0;
    }
  }
}

// Inverse iteration for eigenvalue lam of the tridiagonal (d, e): a pivoted
// LU of T - lam I (factors in the thread's slice of F: four planes of
// `fplane` doubles, entry k of thread t at k * fs + t), three solves from a
// pseudo-random start, each followed by re-orthogonalisation against the
// `nprev` finished vectors Z[:, c0 .. c0+nprev) of the same cluster and
// normalisation.  Result in column `col` of Z (m x m, col-major).
__device__ inline void inverse_iteration(const double* d, const double* e, int m, double lam, double pivtiny,
                                         double* F, int fs, int fplane, double* Z, int col, int c0, int nprev) {
  const int t = threadIdx.x;
  double* u1 = F;                                  // [k * fs + t]
  double* u2 = F + fplane;
  double* u3 = F + 2 * fplane;
  double* L = F + 3 * fplane;
  uint64_t piv[2] = {0ull, 0ull};
  double a = d[0] - lam, c = (m > 1) ? e[0] : 0.0;
  for (int k = 0; k < m - 1; ++k) {
    const double b = e[k], a1 = d[k + 1] - lam, c1 = (k + 1 < m - 1) ? e[k + 1] : 0.0;
    const size_t ix = (size_t)k * fs + t;
    if (fabs(a) >= fabs(b)) {
      const double l = (a != 0.0) ? b / a : 0.0;
      u1[ix] = a; u2[ix] = c; u3[ix] = 0.0; L[ix] = l;
      a = a1 - l * c;
      c = c1;
    } else {
      const double l = a / b;
      piv[k >> 6] |= 1ull << (k & 63);
      u1[ix] = b; u2[ix] = a1; u3[ix] = c1; L[ix] = l;
      a = c - l * a1;
      c = -l * c1;
    }
  }
  u1[(size_t)(m - 1) * fs + t] = a;
  // the back substitutions multiply by the reciprocals of the pivots (each
  // perturbed away from zero): u1 holds 1 / pivot from here on
  for (int k = 0; k < m; ++k) {
    const size_t ix = (size_t)k * fs + t;
    double pv = u1[ix];
    if (fabs(pv) < pivtiny) pv = (pv < 0.0) ? -pivtiny : pivtiny;
    u1[ix] = 1.0 / pv;
  }

  double* x = Z + (size_t)col * m;
  for (int k = 0; k < m; ++k) x[k] = uniform_centered(0x9E3779B97F4A7C15ull + col, (uint64_t)k) * 2.0;
  for (int it = 0; it < 3; ++it) {
    // forward: row interchanges and L
    for (int k = 0; k < m - 1; ++k) {
      const size_t ix = (size_t)k * fs + t;
      if ((piv[k >> 6] >> (k & 63)) & 1ull) {
        const double tmp = x[k];
        x[k] = x[k + 1];
        x[k + 1] = tmp;
      }
      x[k + 1] -= L[ix] * x[k];
    }
    // back substitution with U (reciprocal pivots)
    for (int k = m - 1; k >= 0; --k) {
      const size_t ix = (size_t)k * fs + t;
      double r = x[k];
      if (k + 1 < m) r -= u2[ix] * x[k + 1];
      if (k + 2 < m) r -= u3[ix] * x[k + 2];
      x[k] = r * u1[ix];
    }
    // re-orthogonalise against the cluster's finished vectors, normalise
    for (int q = 0; q < nprev; ++q) {
      const double* zq = Z + (size_t)(c0 + q) * m;
      double s = 0.0;
      for (int k = 0; k < m; ++k) s += zq[k] * x[k];
      for (int k = 0; k < m; ++k) x[k] -= s * zq[k];
    }
    double mx = 0.0;
    for (int k = 0; k < m; ++k) mx = fmax(mx, fabs(x[k]));
    if (!(mx > 0.0)) mx = 1.0;
    const double rmx = 1.0 / mx;
    double s2 = 0.0;
    for (int k = 0; k < m; ++k) {
      x[k] *= rmx;
      s2 += x[k] * x[k];
    }
    const double inv = 1.0 / sqrt(s2);
    for (int k = 0; k < m; ++k) x[k] *= inv;
  }
}

// All eigenpairs of the symmetric tridiagonal (d, e) (e[i] couples i, i+1;
// e2 = e^2), computed by one CTA of NT >= m threads: eigenvalues ascending by
// multisection on Sturm counts (up to 8 lanes each, accurate to ~eps*||T||), then
// eigenvectors (columns of the m x m column-major Z) by inverse iteration,
// clusters (gap <= 1e-3 ||T||_1) handled in rounds with re-orthogonalisation.
// F: inverse-iteration scratch, 4 * kMaxCols * NT doubles of global memory
// (fs = 0), or 4 m^2 doubles of shared memory with fs = m (entry stride m,
// planes of m * m); cl: kMaxCols ints of shared memory; *onenrm (shared)
// receives ||T||_1.  Returns false (block-uniform) when T has non-finite
// entries.  Must be called by all threads of the CTA.
template <int NT, int GMAX = 8>
__device__ bool tridiag_eigen_cta(const double* d, const double* e, const double* e2, int m, double* th, double* Z,
                                  double* F, int* cl, double* onenrm, int fs = 0) {
  __shared__ double sh_glo, sh_ghi, sh_pivmin;
  __shared__ int sh_rounds;
  const int t = threadIdx.x;
  if (t == 0) {
    double glo = d[0], ghi = d[0], nrm = 0.0, emax2 = 0.0, finite = 0.0;
    for (int k = 0; k < m; ++k) {
      const double off = (k > 0 ? fabs(e[k - 1]) : 0.0) + (k < m - 1 ? fabs(e[k]) : 0.0);
      glo = fmin(glo, d[k] - off);
      ghi = fmax(ghi, d[k] + off);
      nrm = fmax(nrm, fabs(d[k]) + off);
      emax2 = fmax(emax2, e2[k]);
      finite += d[k] + off;
    }
    const double pivmin = kSafeMin * fmax(1.0, emax2);
    const double tnorm = fmax(fabs(glo), fabs(ghi));
    sh_glo = glo - 2.0 * kUnitRoundoff * tnorm * m - 2.0 * pivmin;
    sh_ghi = ghi + 2.0 * kUnitRoundoff * tnorm * m + 2.0 * pivmin;
    sh_pivmin = pivmin;
    *onenrm = isfinite(finite) ? nrm : -1.0;
  }
  __syncthreads();
  if (!(*onenrm >= 0.0)) return false;
  // Multisection: eigenvalue i belongs to G consecutive lanes (G a power of
  // two, G m <= NT, at most GMAX), each evaluating kSturmP interior points per
  // round with interleaved Sturm chains (their divisions overlap), so a round
  // cuts the bracket into G kSturmP + 1 pieces.  All G lanes hold the same
  // bracket, updated from the first point whose count exceeds i.
  {
    int G = 1;
    while (G < GMAX && 2 * G * m <= NT) G *= 2;
    const int i = t / G, g = t % G;
    const int np = G * kSturmP;
    const unsigned gmask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << ((t & 31) & ~(G - 1)));
    if (i < m) {
      double lo = sh_glo, hi = sh_ghi;
      for (int it = 0; it < 128; ++it) {
        // The stop test must be the same in every lane of the group (they
        // shuffle below): it reads only the bracket and the round's first and
        // last points, which every lane computes with the same arithmetic,
        // and the group votes on it as well.
        const double x0 = lo + (hi - lo) * (1.0 / (double)(np + 1));
        const double xl = lo + (hi - lo) * ((double)np / (double)(np + 1));
        bool stop = hi - lo <= 2.0 * kUnitRoundoff * fmax(fabs(lo), fabs(hi)) + 4.0 * sh_pivmin || x0 <= lo ||
                    xl >= hi;
        stop = __any_sync(gmask, stop);
        if (stop) break;
        double x[kSturmP];
#pragma unroll
        for (int q = 0; q < kSturmP; ++q) x[q] = lo + (hi - lo) * ((double)(g * kSturmP + q + 1) / (double)(np + 1));
        int cnt[kSturmP];
        sturm_counts<kSturmP>(d, e2, m, x, sh_pivmin, cnt);
        int first = kSturmP;   // the group-local index of this lane's first point with count > i
#pragma unroll
        for (int q = kSturmP - 1; q >= 0; --q)
          if (cnt[q] > i) first = q;
        int f = g * kSturmP + first;   // global index; np when none of this lane's points qualifies
        if (first == kSturmP) f = np;
        for (int o = 1; o < G; o <<= 1) f = min(f, __shfl_xor_sync(gmask, f, o));
        // the bracket's new ends: points f-1 and f of the round (lo / hi at the ends)
        const double nlo = f == 0 ? lo : lo + (hi - lo) * ((double)f / (double)(np + 1));
        const double nhi = f == np ? hi : lo + (hi - lo) * ((double)(f + 1) / (double)(np + 1));
        lo = nlo;
        hi = nhi;
      }
      if (g == 0) th[i] = 0.5 * (lo + hi);
    }
  }
  __syncthreads();
  if (t == 0) {
    const double ortol = 1e-3 * *onenrm;
    int rounds = 1;
    cl[0] = 0;
    for (int i = 1; i < m; ++i) {
      cl[i] = (th[i] - th[i - 1] > ortol) ? i : cl[i - 1];
      rounds = max(rounds, i - cl[i] + 1);
    }
    sh_rounds = rounds;
  }
  __syncthreads();
  const double pivtiny = kUnitRoundoff * fmax(*onenrm, kSafeMin);
  for (int r = 0; r < sh_rounds; ++r) {
    if (t < m && t - cl[t] == r) {
      if (fs > 0) inverse_iteration(d, e, m, th[t], pivtiny, F, fs, m * fs, Z, t, cl[t], r);
      else inverse_iteration(d, e, m, th[t], pivtiny, F, NT, kMaxCols * NT, Z, t, cl[t], r);
    }
    __syncthreads();
  }
  return true;
}

}  // namespace lg
