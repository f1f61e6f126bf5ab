/*
 * irlm_oracle.c — CPU restatement of the reference's implicitly restarted
 * Lanczos eigensolver.  TEST INFRASTRUCTURE ONLY: imported by tests/, by
 * __graft_entry__.smoke() to check results and by bench.py's cpu_baseline /
 * --impl reference leg.  The product path never links or calls it.
 *
 * Follows (reference file:line):
 *   lanczos_extend ............ src/irlm_lanczos.cu:110-148
 *   cgs_orthogonalize ......... src/lanczos_ops.cuh:113-132
 *   dgks_reorth ............... src/lanczos_ops.cuh:147-192 (threshold 1/sqrt2,
 *                               at most two refinement passes, then rnorm = 0)
 *   safe_scale ................ src/lanczos_ops.cuh:204-216
 *   inject_random_restart ..... src/lanczos_ops.cuh:229-253
 *   adaptive_breakdown_tol .... src/lanczos_ops.cuh:264-277
 *   irlm restart loop ......... src/irlm_lanczos.cu:225-363
 *   givens / bulge chase ...... src/tridiag.cuh:33-124
 *   Ritz vectors .............. src/lanczos_ops.cuh:318-338
 * with these deliberate changes, which the CUDA engine shares:
 *   - LAPACK dstev (src/tridiag.cuh:138-163) is replaced by an implicit
 *     symmetric QR with Wilkinson shift (Golub & Van Loan 8.3), since no
 *     LAPACK is linked here;
 *   - wanted-set ordering, convergence test tol*max(eps^(2/3), |theta|), zero
 *     bound locking and the NEV adjustment follow ARPACK (dsgets, dsconv,
 *     dsaup2), so which = LM/SM/LA/SA/BE all work (the reference only keeps the
 *     smallest algebraic values and uses tol*max(|theta|, DBL_MIN));
 *   - after an invariant subspace the coupling beta is set to 0 (ARPACK dgetv0)
 *     instead of the norm of the random vector;
 *   - cgs2 != 0 applies the second Gram-Schmidt pass unconditionally (as the
 *     CUDA engine does); cgs2 == 0 keeps the reference's conditional DGKS.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define DGKS 0.7071067811865476
#define UNIT 1.1102230246251565e-16          /* 2^-53 */
#define EPS23_ARPACK 2.3112508282095347e-11  /* (2^-53)^(2/3) */
#define EPS23_REF 3.6687695461231177e-11     /* DBL_EPSILON^(2/3) */

enum { LM = 0, SM = 1, LA = 2, SA = 3, BE = 4 };

typedef struct {
  int n;
  const int *rp, *ci;
  const double *va;
} csr_t;

static void spmv(const csr_t *A, const double *x, double *y) {
  int i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < A->n; ++i) {
    double s = 0.0;
    for (int k = A->rp[i]; k < A->rp[i + 1]; ++k) s += A->va[k] * x[A->ci[k]];
    y[i] = s;
  }
}

static double dot(int n, const double *a, const double *b) {
  double s = 0.0;
  int i;
#pragma omp parallel for reduction(+ : s) schedule(static)
  for (i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* h[0..nc) = V[:, 0..nc)^T x   (V column-major, ld = n) */
static void gemv_t(int n, int nc, const double *V, const double *x, double *h) {
  for (int c = 0; c < nc; ++c) h[c] = 0.0;
#pragma omp parallel
  {
    double loc[256];
    for (int c = 0; c < nc; ++c) loc[c] = 0.0;
    int i;
#pragma omp for schedule(static)
    for (i = 0; i < n; ++i) {
      const double xi = x[i];
      for (int c = 0; c < nc; ++c) loc[c] += V[(size_t)c * n + i] * xi;
    }
#pragma omp critical
    for (int c = 0; c < nc; ++c) h[c] += loc[c];
  }
}

/* y -= V[:, 0..nc) h */
static void gemv_n_sub(int n, int nc, const double *V, const double *h, double *y) {
  int i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < n; ++i) {
    double s = 0.0;
    for (int c = 0; c < nc; ++c) s += V[(size_t)c * n + i] * h[c];
    y[i] -= s;
  }
}

static void scale(int n, double *x, double s) {
  int i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < n; ++i) x[i] *= s;
}

static void safe_scale(int n, double *v, double rnorm) {
  if (rnorm >= DBL_MIN) scale(n, v, 1.0 / rnorm);
  else if (rnorm > 0.0) {
    scale(n, v, DBL_MIN / rnorm);
    scale(n, v, 1.0 / DBL_MIN);
  }
}

static double breakdown_tol(const double *alpha, const double *beta, int j) {
  double est = 0.0;
  for (int i = 0; i <= j; ++i) {
    double rs = fabs(alpha[i]);
    if (i > 0) rs += fabs(beta[i]);
    if (i < j) rs += fabs(beta[i + 1]);
    if (rs > est) est = rs;
  }
  return EPS23_REF * (est > DBL_MIN ? est : DBL_MIN);
}

static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

typedef struct {
  int n, m;
  double *V, *w, *r, *h;
  double *alpha, *beta;
  int cgs2;
  long long reorths, pass3, breakdowns;
  uint64_t seed;
} lz_t;

/* Lanczos steps j = start .. end-1; beta[j+1] = ||r||, V[:, j+1] = r/||r||. */
static void extend(lz_t *L, const csr_t *A, int start, int end) {
  const int n = L->n;
  for (int j = start; j < end; ++j) {
    double *vj = L->V + (size_t)j * n;
    spmv(A, vj, L->w);
    const double wnorm = sqrt(dot(n, L->w, L->w));
    /* CGS pass */
    gemv_t(n, j + 1, L->V, L->w, L->h);
    memcpy(L->r, L->w, sizeof(double) * n);
    gemv_n_sub(n, j + 1, L->V, L->h, L->r);
    double a = L->h[j];
    double rnorm = sqrt(dot(n, L->r, L->r));
    /* DGKS refinement */
    if (L->cgs2 || rnorm <= DGKS * wnorm) {
      for (int pass = 0; pass < 2; ++pass) {
        ++L->reorths;
        if (pass == 1) ++L->pass3;
        gemv_t(n, j + 1, L->V, L->r, L->h);
        gemv_n_sub(n, j + 1, L->V, L->h, L->r);
        a += L->h[j];
        const double rn = sqrt(dot(n, L->r, L->r));
        if (rn > DGKS * rnorm) { rnorm = rn; break; }
        if (pass == 1) { rnorm = 0.0; break; }
        rnorm = rn;
      }
    }
    L->alpha[j] = a;
    double bnext = rnorm;
    if (rnorm < breakdown_tol(L->alpha, L->beta, j)) {
      /* invariant subspace: random vector orthogonal to V[:, 0..j] */
      ++L->breakdowns;
      for (int i = 0; i < n; ++i) {
        uint64_t z = mix64(L->seed * 0x100000001B3ull + mix64(((uint64_t)j << 32) + (uint64_t)i + 77));
        L->r[i] = (double)(z >> 11) * (1.0 / 9007199254740992.0) - 0.5;
      }
      for (int pass = 0; pass < 2; ++pass) {
        gemv_t(n, j + 1, L->V, L->r, L->h);
        gemv_n_sub(n, j + 1, L->V, L->h, L->r);
      }
      rnorm = sqrt(dot(n, L->r, L->r));
      bnext = 0.0;
    }
    L->beta[j + 1] = bnext;
    double *vn = L->V + (size_t)(j + 1) * n;
    memcpy(vn, L->r, sizeof(double) * n);
    if (rnorm > 0.0) safe_scale(n, vn, rnorm);
  }
}

/* [c -s; s c][a; b] = [r; 0] */
static void givens(double a, double b, double *c, double *s) {
  if (b == 0.0) { *c = 1.0; *s = 0.0; }
  else if (fabs(b) > fabs(a)) { double t = -a / b; *s = 1.0 / sqrt(1.0 + t * t); *c = *s * t; }
  else { double t = -b / a; *c = 1.0 / sqrt(1.0 + t * t); *s = *c * t; }
}

/* One implicit QR sweep with shift sigma on block [l, mm]; rotations applied
 * to the columns of M (m x m column-major) when M != NULL. */
static void chase(double *d, double *e, int l, int mm, double sigma, double *M, int m) {
  double bulge = 0.0;
  for (int k = l; k < mm; ++k) {
    double c, s;
    if (k == l) givens(d[l] - sigma, e[l], &c, &s);
    else { givens(e[k - 1], bulge, &c, &s); e[k - 1] = c * e[k - 1] - s * bulge; }
    const double dk = d[k], dk1 = d[k + 1], ek = e[k];
    const double cc = c * c, ss = s * s, cs = c * s;
    d[k] = cc * dk - 2.0 * cs * ek + ss * dk1;
    d[k + 1] = ss * dk + 2.0 * cs * ek + cc * dk1;
    e[k] = cs * (dk - dk1) + (cc - ss) * ek;
    if (k + 1 < mm) { bulge = -s * e[k + 1]; e[k + 1] = c * e[k + 1]; }
    if (M) {
      for (int i = 0; i < m; ++i) {
        const double a = M[i + (size_t)k * m], b = M[i + (size_t)(k + 1) * m];
        M[i + (size_t)k * m] = c * a - s * b;
        M[i + (size_t)(k + 1) * m] = s * a + c * b;
      }
    }
  }
}

/* eigen-decomposition of the symmetric tridiagonal (d, e); Z = eigenvectors */
static int tridiag_eig(int m, double *d, double *e, double *Z) {
  for (int i = 0; i < m * m; ++i) Z[i] = 0.0;
  for (int i = 0; i < m; ++i) Z[i + (size_t)i * m] = 1.0;
  int sweeps = 0;
  for (;;) {
    for (int i = 0; i < m - 1; ++i)
      if (e[i] != 0.0 && e[i] * e[i] <= UNIT * UNIT * fabs(d[i]) * fabs(d[i + 1]) + DBL_MIN) e[i] = 0.0;
    int mm = m - 1;
    while (mm > 0 && e[mm - 1] == 0.0) --mm;
    if (mm == 0) return 0;
    if (++sweeps > 30 * m) return -1;
    int l = mm - 1;
    while (l > 0 && e[l - 1] != 0.0) --l;
    const double aa = d[mm - 1], cc = d[mm], bb = e[mm - 1];
    const double delta = 0.5 * (aa - cc);
    const double den = delta + copysign(hypot(delta, bb), delta == 0.0 ? 1.0 : delta);
    const double mu = (den != 0.0) ? cc - bb * (bb / den) : cc - fabs(bb);
    chase(d, e, l, mm, mu, Z, m);
  }
}

static void swap3(double *rz, double *bd, int *id, int i, int k) {
  double t = rz[i]; rz[i] = rz[k]; rz[k] = t;
  t = bd[i]; bd[i] = bd[k]; bd[k] = t;
  int u = id[i]; id[i] = id[k]; id[k] = u;
}

static void sort_ascending(int m, double *rz, double *bd, int *id) {
  for (int i = 1; i < m; ++i)
    for (int k = i; k > 0 && rz[k - 1] > rz[k]; --k) swap3(rz, bd, id, k - 1, k);
}

/* ARPACK dsgets ordering: wanted values last. Input ascending. */
static void order_wanted(int which, int m, int nev, double *rz, double *bd, int *id) {
  if (which == SA) {
    for (int i = 0; i < m / 2; ++i) swap3(rz, bd, id, i, m - 1 - i);
  } else if (which == LM || which == SM) {
    for (int i = 1; i < m; ++i)
      for (int k = i; k > 0; --k) {
        const double a = fabs(rz[k - 1]), b = fabs(rz[k]);
        if (!((which == LM) ? (a > b) : (a < b))) break;
        swap3(rz, bd, id, k - 1, k);
      }
  } else if (which == BE) {
    const int np = m - nev, kevd2 = nev / 2;
    if (nev > 1) {
      const int cnt = kevd2 < np ? kevd2 : np, off = kevd2 > np ? kevd2 : np;
      for (int i = 0; i < cnt; ++i) swap3(rz, bd, id, i, off + i);
    }
  }
}

/*
 * Returns 0 converged, 1 not converged (limit), <0 error.
 * info[0] nconv, info[1] restarts, info[2] steps, info[3] reorth passes,
 * info[4] breakdowns.  alpha0/beta0 (optional, m and m+1 entries) receive the
 * tridiagonal of the first m-step factorisation.
 */
int oracle_irlm(int n, const int *rowptr, const int *colidx, const double *vals, int k, int m, int which,
                double tol, int maxiter, long long max_steps, const double *v0, uint64_t seed, int cgs2,
                double *evals, double *evecs, long long *info, double *alpha0, double *beta0) {
  if (k < 1 || k >= n || m <= k || m > n || m > 255) return -1;
  csr_t A = {n, rowptr, colidx, vals};
  lz_t L;
  memset(&L, 0, sizeof(L));
  L.n = n;
  L.m = m;
  L.cgs2 = cgs2;
  L.seed = seed;
  L.V = (double *)calloc((size_t)n * (m + 1), sizeof(double));
  L.w = (double *)malloc(sizeof(double) * n);
  L.r = (double *)malloc(sizeof(double) * n);
  L.h = (double *)malloc(sizeof(double) * (m + 2));
  L.alpha = (double *)calloc(m + 2, sizeof(double));
  L.beta = (double *)calloc(m + 2, sizeof(double));
  double *d = (double *)malloc(sizeof(double) * m), *e = (double *)malloc(sizeof(double) * m);
  double *Z = (double *)malloc(sizeof(double) * m * m), *Q = (double *)malloc(sizeof(double) * m * m);
  double *rz = (double *)malloc(sizeof(double) * m), *bd = (double *)malloc(sizeof(double) * m);
  double *shifts = (double *)malloc(sizeof(double) * m);
  int *id = (int *)malloc(sizeof(int) * m);
  double *Vn = (double *)malloc(sizeof(double) * (size_t)n * (m + 1));
  int ret = 0;
  if (!maxiter) maxiter = 10 * n;
  if (tol <= 0.0) tol = UNIT;

  /* starting vector */
  if (v0) memcpy(L.V, v0, sizeof(double) * n);
  else
    for (int i = 0; i < n; ++i) {
      uint64_t z = mix64(seed * 0x100000001B3ull + mix64((uint64_t)i));
      L.V[i] = (double)(z >> 11) * (1.0 / 9007199254740992.0) - 0.5;
    }
  safe_scale(n, L.V, sqrt(dot(n, L.V, L.V)));

  extend(&L, &A, 0, m);
  long long steps = m;
  if (alpha0) memcpy(alpha0, L.alpha, sizeof(double) * m);
  if (beta0) memcpy(beta0, L.beta, sizeof(double) * (m + 1));

  int iter = 1, nconv = 0;
  for (;;) {
    const double bn = L.beta[m];
    for (int i = 0; i < m; ++i) { d[i] = L.alpha[i]; e[i] = (i < m - 1) ? L.beta[i + 1] : 0.0; }
    if (tridiag_eig(m, d, e, Z) != 0) { ret = -5; goto out; }
    for (int i = 0; i < m; ++i) id[i] = i;
    for (int i = 0; i < m; ++i) rz[i] = d[i];
    for (int i = 0; i < m; ++i) bd[i] = 0.0;
    sort_ascending(m, rz, bd, id);
    for (int i = 0; i < m; ++i) bd[i] = fabs(bn * Z[(m - 1) + (size_t)id[i] * m]);

    int nev = k, np = m - k;
    order_wanted(which, m, nev, rz, bd, id);
    nconv = 0;
    for (int i = np; i < m; ++i)
      if (bd[i] <= tol * fmax(EPS23_ARPACK, fabs(rz[i]))) ++nconv;
    const int np0 = np;
    for (int i = 0; i < np0; ++i)
      if (bd[i] == 0.0) { --np; ++nev; }
    const int done = (nconv >= k) || (iter > maxiter) || (np == 0) || (max_steps > 0 && steps >= max_steps);
    if (done) {
      const int off = m - k;
      sort_ascending(k, rz + off, bd + off, id + off);
      for (int c = 0; c < k; ++c) evals[c] = rz[off + c];
      if (evecs) {
        int i;
#pragma omp parallel for schedule(static)
        for (i = 0; i < n; ++i)
          for (int c = 0; c < k; ++c) {
            double s = 0.0;
            const double *zc = Z + (size_t)id[off + c] * m;
            for (int q = 0; q < m; ++q) s += L.V[(size_t)q * n + i] * zc[q];
            evecs[(size_t)c * n + i] = s;
          }
      }
      ret = (nconv >= k) ? 0 : 1;
      break;
    }
    /* NEV adjustment (ARPACK dsaup2) */
    const int nevbef = nev;
    nev += (nconv < np / 2 ? nconv : np / 2);
    if (nev == 1 && m >= 6) nev = m / 2;
    else if (nev == 1 && m > 2) nev = 2;
    np = m - nev;
    if (nevbef < nev) {
      sort_ascending(m, rz, bd, id);
      order_wanted(which, m, nev, rz, bd, id);
    }
    for (int i = 0; i < np; ++i) shifts[i] = rz[i];
    for (int i = 1; i < np; ++i)
      for (int q = i; q > 0 && bd[q - 1] < bd[q]; --q) {
        double u = bd[q - 1]; bd[q - 1] = bd[q]; bd[q] = u;
        u = shifts[q - 1]; shifts[q - 1] = shifts[q]; shifts[q] = u;
      }
    /* exact shifts by bulge chasing (ARPACK dsapps, with deflation splits) */
    for (int i = 0; i < m; ++i) { d[i] = L.alpha[i]; e[i] = (i < m - 1) ? L.beta[i + 1] : 0.0; }
    for (int i = 0; i < m * m; ++i) Q[i] = 0.0;
    for (int i = 0; i < m; ++i) Q[i + (size_t)i * m] = 1.0;
    for (int is = 0; is < np; ++is) {
      int istart = 0;
      while (istart < m - 1) {
        int iend = m - 1;
        for (int i = istart; i < m - 1; ++i)
          if (fabs(e[i]) <= UNIT * (fabs(d[i]) + fabs(d[i + 1]))) { e[i] = 0.0; iend = i; break; }
        if (istart < iend) chase(d, e, istart, iend, shifts[is], Q, m);
        istart = iend + 1;
      }
    }
    for (int i = 0; i < m - 1; ++i)
      if (fabs(e[i]) <= UNIT * (fabs(d[i]) + fabs(d[i + 1]))) e[i] = 0.0;
    /* V_new = V Q[:, 0..nev], residual r = Q[m-1, nev-1] f + e[nev-1] V_new[:, nev] */
    {
      const double rcoef = bn * Q[(m - 1) + (size_t)(nev - 1) * m];
      const double tau = (nev < m) ? e[nev - 1] : 0.0;
      int i;
#pragma omp parallel for schedule(static)
      for (i = 0; i < n; ++i) {
        for (int c = 0; c <= nev; ++c) {
          double s = 0.0;
          for (int q = 0; q < m; ++q) s += L.V[(size_t)q * n + i] * Q[q + (size_t)c * m];
          Vn[(size_t)c * n + i] = s;
        }
        L.r[i] = rcoef * L.V[(size_t)m * n + i] + tau * Vn[(size_t)nev * n + i];
      }
      memcpy(L.V, Vn, sizeof(double) * (size_t)n * nev);
    }
    for (int i = 0; i < m; ++i) L.alpha[i] = (i < nev) ? d[i] : 0.0;
    for (int i = 1; i <= m + 1; ++i) {
      if (i < nev) L.beta[i] = e[i - 1];
      else if (i > nev) L.beta[i] = 0.0;
    }
    double rn = sqrt(dot(n, L.r, L.r));
    if (rn < breakdown_tol(L.alpha, L.beta, nev - 1)) {
      ++L.breakdowns;
      for (int i = 0; i < n; ++i) {
        uint64_t z = mix64(L.seed * 0x100000001B3ull + mix64(((uint64_t)(nev + 1000) << 32) + (uint64_t)i));
        L.r[i] = (double)(z >> 11) * (1.0 / 9007199254740992.0) - 0.5;
      }
      for (int pass = 0; pass < 2; ++pass) {
        gemv_t(n, nev, L.V, L.r, L.h);
        gemv_n_sub(n, nev, L.V, L.h, L.r);
      }
      rn = sqrt(dot(n, L.r, L.r));
      L.beta[nev] = 0.0;
    } else {
      L.beta[nev] = rn;
    }
    memcpy(L.V + (size_t)nev * n, L.r, sizeof(double) * n);
    safe_scale(n, L.V + (size_t)nev * n, rn);
    extend(&L, &A, nev, m);
    steps += m - nev;
    ++iter;
  }
out:
  if (info) {
    info[0] = nconv;
    info[1] = iter - 1;
    info[2] = steps;
    info[3] = L.reorths;
    info[4] = L.breakdowns;
  }
  free(L.V); free(L.w); free(L.r); free(L.h); free(L.alpha); free(L.beta);
  free(d); free(e); free(Z); free(Q); free(rz); free(bd); free(shifts); free(id); free(Vn);
  return ret;
}

/* Lanczos steps only (no restarts): n_steps steps from v0 on the matrix, used
 * to time the CPU reference as Lanczos steps per second on a bounded sample.
 * Returns the number of steps done. */
long long oracle_lanczos_steps(int n, const int *rowptr, const int *colidx, const double *vals, int m,
                               const double *v0, int cgs2, double *alpha, double *beta) {
  csr_t A = {n, rowptr, colidx, vals};
  lz_t L;
  memset(&L, 0, sizeof(L));
  L.n = n;
  L.m = m;
  L.cgs2 = cgs2;
  L.seed = 7;
  L.V = (double *)calloc((size_t)n * (m + 1), sizeof(double));
  L.w = (double *)malloc(sizeof(double) * n);
  L.r = (double *)malloc(sizeof(double) * n);
  L.h = (double *)malloc(sizeof(double) * (m + 2));
  L.alpha = (double *)calloc(m + 2, sizeof(double));
  L.beta = (double *)calloc(m + 2, sizeof(double));
  memcpy(L.V, v0, sizeof(double) * n);
  safe_scale(n, L.V, sqrt(dot(n, L.V, L.V)));
  extend(&L, &A, 0, m);
  if (alpha) memcpy(alpha, L.alpha, sizeof(double) * m);
  if (beta) memcpy(beta, L.beta, sizeof(double) * (m + 1));
  free(L.V); free(L.w); free(L.r); free(L.h); free(L.alpha); free(L.beta);
  return m;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Threads of the parallel loops started by the calling thread (all host cores
 * by default; a launcher may have set OMP_NUM_THREADS=1).  Returns the count
 * now in effect. */
int oracle_set_num_threads(int nth) {
#ifdef _OPENMP
  if (nth > 0) omp_set_num_threads(nth);
  return omp_get_max_threads();
#else
  (void)nth;
  return 1;
#endif
}
