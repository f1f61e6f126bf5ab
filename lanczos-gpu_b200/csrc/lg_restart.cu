// lg_restart.cu — the implicit-restart step of IRLM, on the device, in one CTA.
//
// Reference: src/irlm_lanczos.cu:225-363 (host loop: LAPACK dstev, convergence
// test, NEV adjustment, exact shifts, bulge chase, H2D of Q) and
// src/tridiag.cuh:33-124 (givens, apply_shifts_tridiag).  Everything runs in
// one CTA so the host never touches the tridiagonal, and every phase that can
// be parallel is:
//
//   1. beta_m = ||r|| from the partial sums of the last Gram-Schmidt pass,
//      DGKS / breakdown checks for the last step;
//   2. Ritz values: multisection on Sturm counts, a few lanes per eigenvalue
//      (all eigenvalues to ~eps*||T|| absolute accuracy, the accuracy of QR);
//   3. eigenvectors of T: inverse iteration with a pivoted tridiagonal LU,
//      one thread per eigenvalue, vectors of eigenvalue clusters
//      (gap <= 1e-3 ||T||) re-orthogonalised in rounds (the method of LAPACK
//      dstein);
//   4. Ritz estimates |beta_m * z_last,i|, ARPACK-style ordering of the wanted
//      end of the spectrum for which = LM/SM/LA/SA/BE, convergence test
//      |bound| <= tol * max(eps^(2/3), |theta|), locking of zero bounds and
//      the NEV adjustment of ARPACK's dsaup2;
//   5. either the wanted pairs are selected (finished), or the np exact shifts
//      are applied by bulge chasing.  Up to 32 bulges run at once, one lane
//      each, three rows apart (rotations of neighbouring bulges then touch
//      disjoint entries), and the step's rotations are applied to Q by several
//      threads per row, each taking a share of them.  The result equals the shift-after-shift chase of the
//      reference; the deflation splitting of ARPACK's dsapps is not done
//      (a negligible coupling just makes the chase pass identity rotations).
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_tridiag.cuh"

#include <cmath>

namespace lg {

namespace {

constexpr int kRsThreads = 512;   // bisection lanes per eigenvalue and Q-update threads per row scale with it
constexpr int kRsSmemM = 72;   // m <= 72: M and the 4 m^2 inverse-iteration factors (5 m^2 doubles) fit in shared memory
constexpr double kUnit = 1.1102230246251565e-16;        // 2^-53
constexpr double kEps23Arpack = 2.3112508282095347e-11;  // (2^-53)^(2/3)

// Order (rz, bd, id) so that the nev wanted values are at the end
// (ARPACK dsgets restated: LA ascending, SA descending, LM ascending |x|,
// SM descending |x|, BE ascending then the low end swapped in front of the
// high end).  Input arrays are in ascending value order.
__device__ void order_wanted(int which, int m, int nev, double* rz, double* bd, int* id) {
  auto swap3 = [&](int i, int k) {
    double t = rz[i]; rz[i] = rz[k]; rz[k] = t;
    t = bd[i]; bd[i] = bd[k]; bd[k] = t;
    int u = id[i]; id[i] = id[k]; id[k] = u;
  };
  if (which == WHICH_SA) {
    for (int i = 0; i < m / 2; ++i) swap3(i, m - 1 - i);
  } else if (which == WHICH_LM || which == WHICH_SM) {
    for (int i = 1; i < m; ++i) {
      for (int k = i; k > 0; --k) {
        const double a = fabs(rz[k - 1]), b = fabs(rz[k]);
        const bool out = (which == WHICH_LM) ? (a > b) : (a < b);
        if (!out) break;
        swap3(k - 1, k);
      }
    }
  } else if (which == WHICH_BE) {
    const int np = m - nev, kevd2 = nev / 2;
    if (nev > 1) {
      const int cnt = kevd2 < np ? kevd2 : np;
      const int off = kevd2 > np ? kevd2 : np;
      for (int i = 0; i < cnt; ++i) swap3(i, off + i);
    }
  }
}

__device__ void sort_ascending(int lo, int hi, double* rz, double* bd, int* id) {
  for (int i = lo + 1; i < hi; ++i)
    for (int k = i; k > lo && rz[k - 1] > rz[k]; --k) {
      double u = rz[k - 1]; rz[k - 1] = rz[k]; rz[k] = u;
      u = bd[k - 1]; bd[k - 1] = bd[k]; bd[k] = u;
      const int w = id[k - 1]; id[k - 1] = id[k]; id[k] = w;
    }
}

}  // namespace

__global__ void __launch_bounds__(kRsThreads, 1) restart_kernel(RestartArgs a) {
  int* state = a.state;
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(16) double M[];   // m x m, column-major
  __shared__ double d[kMaxCols], e[kMaxCols], e2[kMaxCols], th[kMaxCols];
  __shared__ double rz[kMaxCols], bd[kMaxCols], shifts[kMaxCols];
  __shared__ double rot_c[2][2][32], rot_s[2][2][32];
  __shared__ int rot_k[2][2][32];
  __shared__ int id[kMaxCols], cl[kMaxCols];
  __shared__ double sh_bn, sh_onenrm;
  __shared__ int sh_stop, sh_done, sh_nev, sh_np, sh_nconv;

  const int t = threadIdx.x, m = a.m, lane = t & 31;

  // ---- 1. residual norm and checks for the last step -----------------------
  if (t < 32) {
    double nrm2 = 0.0;
    for (int r = t; r < a.nrows_in; r += 32) nrm2 += a.part_in[(size_t)r * kPartStride + kPartScalar];
    nrm2 = warp_sum(nrm2);
    if (t == 0) {
      const double bn = sqrt(nrm2);
      int stop = STATUS_RUNNING;
      if (a.skip_checks) {
        // residual is exactly zero by construction
      } else if (nrm2 <= 0.5 * a.scal[SC_R1N2]) {
        stop = STATUS_PASS3;
      } else {
        double est = 0.0;
        for (int i = 0; i < m; ++i) {
          double rs = fabs(a.alpha[i]);
          if (i > 0) rs += fabs(a.beta[i]);
          if (i < m - 1) rs += fabs(a.beta[i + 1]);
          est = fmax(est, rs);
        }
        if (bn < 3.6687695461231177e-11 * fmax(est, kSafeMin)) stop = STATUS_BREAKDOWN;
      }
      if (stop != STATUS_RUNNING) {
        state[ST_STEP] = m - 1;
        state[ST_STATUS] = stop;
      } else {
        a.beta[m] = bn;
        a.scal[SC_BN] = bn;
      }
      sh_bn = bn;
      sh_stop = stop;
    }
  }
  if (t < m) {
    d[t] = a.alpha[t];
    e[t] = (t < m - 1) ? a.beta[t + 1] : 0.0;
    e2[t] = e[t] * e[t];
  }
  __syncthreads();
  if (sh_stop != STATUS_RUNNING) return;
  const double bn = sh_bn;

  // ---- 2./3. Ritz values (bisection) and eigenvectors of T (inverse iteration);
  // the LU factors of the inverse iterations in shared memory behind M when
  // they fit (their loads sit on the iterations' dependent chains)
  const bool f_smem = m <= kRsSmemM;
  // Two lanes per eigenvalue (eight interior points per round, 17 rounds to
  // full precision).  Fewer points per round take more rounds of the
  // dependent Sturm chains; more points cost more FP64 work on this one SM.
  // Measured at m = 60 (cycles of this phase): 1 lane 267 k, 2 lanes 183 k,
  // 4 lanes 199 k, 8 lanes 249 k.
  if (!tridiag_eigen_cta<kRsThreads, 2>(d, e, e2, m, th, M, f_smem ? M + (size_t)m * m : a.scratch, cl, &sh_onenrm,
                                        f_smem ? m : 0)) {
    if (t == 0) {
      state[ST_ERRINFO] = 1;
      state[ST_STATUS] = STATUS_TRIDIAG_FAIL;
    }
    return;
  }

  // ---- 4. ordering, Ritz estimates, convergence, NEV adjustment -------------
  if (t == 0) {
    for (int i = 0; i < m; ++i) {
      id[i] = i;
      rz[i] = th[i];
      bd[i] = fabs(bn * M[(m - 1) + (size_t)i * m]);
    }
    const double tol = a.tol > 0.0 ? a.tol : kUnit;
    int nev = a.nev0, np = m - a.nev0;
    order_wanted(a.which, m, nev, rz, bd, id);
    int nconv = 0;
    for (int i = np; i < m; ++i)
      if (bd[i] <= tol * fmax(kEps23Arpack, fabs(rz[i]))) ++nconv;
    const int np0 = np;
    for (int i = 0; i < np0; ++i)
      if (bd[i] == 0.0) { --np; ++nev; }
    const int done = (nconv >= a.nev0) || (a.iter > a.maxiter) || (np == 0) || a.force_done;
    if (!done) {
      const int nevbef = nev;
      nev = nev + (nconv < np / 2 ? nconv : np / 2);
      if (nev == 1 && m >= 6) nev = m / 2;
      else if (nev == 1 && m > 2) nev = 2;
      np = m - nev;
      if (nevbef < nev) {
        sort_ascending(0, m, rz, bd, id);
        order_wanted(a.which, m, nev, rz, bd, id);
      }
    }
    sh_done = done;
    sh_nev = nev;
    sh_np = np;
    sh_nconv = nconv;
  }
  __syncthreads();
  if (!sh_done && t < sh_np) {
    // shifts: the unwanted values rz[0, np), largest Ritz estimate first, ties
    // in their order (a stable sort): thread t places its value by its rank
    const int np = sh_np;
    const double bt = bd[t];
    int rank = 0;
    for (int i = 0; i < np; ++i) {
      const double bi = bd[i];
      rank += (bi > bt) || (bi == bt && i < t);
    }
    shifts[rank] = rz[t];
  }
  __syncthreads();

  if (sh_done) {
    // ---- 5a. wanted Ritz pairs, ascending ----------------------------------
    const int k = a.nev0, off = m - k;
    if (t == 0) {
      sort_ascending(off, m, rz, bd, id);
      const double tol = a.tol > 0.0 ? a.tol : kUnit;
      for (int i = 0; i < k; ++i) {
        a.ritz_out[i] = rz[off + i];
        a.bounds_out[i] = bd[off + i];
        a.conv_out[i] = bd[off + i] <= tol * fmax(kEps23Arpack, fabs(rz[off + i])) ? 1 : 0;
      }
      state[ST_NCONV] = sh_nconv;
      state[ST_KSEL] = k;
      state[ST_NEV_USE] = sh_nev;
      state[ST_DONE] = 1;
    }
    __syncthreads();
    for (int c = 0; c < k; ++c)
      if (t < m) a.zsel[t + (size_t)c * m] = M[t + (size_t)id[off + c] * m];
    return;
  }

  // ---- 5b. exact shifts: pipelined bulge chases ------------------------------
  // T first splits at negligible couplings (an invariant subspace met earlier
  // leaves an exact zero); as in ARPACK's dsapps every shift is applied to
  // every unreduced block.  Couplings that become negligible during the
  // chases are left alone (the bulge then just passes identity rotations).
  const int np = sh_np, nev = sh_nev;
  // Warp 0 computes the rotations of the chase while the other warps apply
  // the rotations computed before to Q (double-buffered rotation lists).
  int tpr = 1;   // threads per row of Q in the rotation updates (warps 1..)
  while (tpr < 32 && 2 * tpr * m <= kRsThreads - 32) tpr *= 2;
  __shared__ int blk_lo[kMaxCols], blk_hi[kMaxCols];
  __shared__ int sh_nblk;
  __syncthreads();   // M (eigenvectors) no longer needed
  for (int i = t; i < m * m; i += kRsThreads) M[i] = ((i % m) == (i / m)) ? 1.0 : 0.0;
  if (t == 0) {
    int nblk = 0, lo = 0;
    for (int i = 0; i < m - 1; ++i) {
      if (fabs(e[i]) <= kUnit * (fabs(d[i]) + fabs(d[i + 1]))) {
        e[i] = 0.0;
        if (i > lo) { blk_lo[nblk] = lo; blk_hi[nblk] = i; ++nblk; }
        lo = i + 1;
      }
    }
    if (m - 1 > lo) { blk_lo[nblk] = lo; blk_hi[nblk] = m - 1; ++nblk; }
    sh_nblk = nblk;
  }
  __syncthreads();
  for (int ib = 0; ib < sh_nblk; ++ib) {
    const int bs = blk_lo[ib], be = blk_hi[ib];   // block rows bs..be (be > bs)
    for (int b0 = 0; b0 < np; b0 += 32) {
      const int nb = min(32, np - b0);
      const int steps = (be - bs) + 3 * (nb - 1);
      double bulge = 0.0;                       // lane's bulge (warp 0)
      const double sigma = (t < 32 && lane < nb) ? shifts[b0 + lane] : 0.0;
      // Steps run in pairs.  Warp 0 computes the rotations of steps 2p and
      // 2p + 1 (a __syncwarp between them: a bulge's next rotation reads the
      // coupling its upper neighbour's rotation has just written) while the
      // other warps apply the previous pair to Q.  Within a pair a bulge's
      // two rotations touch columns k .. k+2 and the next bulge's k-3 .. k-1,
      // so each thread applies both rotations of its bulges in order, and
      // every column of Q receives its rotations in the same order as one
      // step at a time (bitwise the same Q), with half the barriers.
      const int npairs = (steps + 1) / 2;
      for (int pr = 0; pr <= npairs; ++pr) {
        const int buf = pr & 1;
        if (t < 32) {
          if (pr < npairs) {
            for (int q = 0; q < 2; ++q) {
              const int st = 2 * pr + q;
              const int k = bs + st - 3 * lane;
              int kk = -1;
              if (st < steps && lane < nb && k >= bs && k < be) {
                double c, s;
                if (k == bs) {
                  givens(d[bs] - sigma, e[bs], c, s);
                } else {
                  givens(e[k - 1], bulge, c, s);
                  e[k - 1] = c * e[k - 1] - s * bulge;
                }
                const double dk = d[k], dk1 = d[k + 1], ek = e[k];
                const double cc = c * c, ss = s * s, cs = c * s;
                d[k] = cc * dk - 2.0 * cs * ek + ss * dk1;
                d[k + 1] = ss * dk + 2.0 * cs * ek + cc * dk1;
                e[k] = cs * (dk - dk1) + (cc - ss) * ek;
                if (k + 1 < be) {
                  bulge = -s * e[k + 1];
                  e[k + 1] = c * e[k + 1];
                }
                rot_c[buf][q][lane] = c;
                rot_s[buf][q][lane] = s;
                kk = k;
              }
              rot_k[buf][q][lane] = kk;
              __syncwarp();
            }
          }
        } else if (pr > 0 && t - 32 < tpr * m) {
          // the previous pair: the tpr threads of a row split the bulges
          const int tq = t - 32, pb = buf ^ 1;
          const int row = tq / tpr;
          for (int s = tq % tpr; s < nb; s += tpr)
            for (int q = 0; q < 2; ++q) {
              const int k = rot_k[pb][q][s];
              if (k < 0) continue;
              const double c = rot_c[pb][q][s], sn = rot_s[pb][q][s];
              const double x0 = M[row + (size_t)k * m], x1 = M[row + (size_t)(k + 1) * m];
              M[row + (size_t)k * m] = c * x0 - sn * x1;
              M[row + (size_t)(k + 1) * m] = sn * x0 + c * x1;
            }
        }
        __syncthreads();
      }
    }
  }
  if (t == 0)
    for (int i = 0; i < m - 1; ++i)
      if (fabs(e[i]) <= kUnit * (fabs(d[i]) + fabs(d[i + 1]))) e[i] = 0.0;
  __syncthreads();

  // outputs: Q[:, 0..nev], new T, restart residual coefficients
  for (int c = 0; c <= nev && c < m; ++c)
    if (t < m) a.Q[t + (size_t)c * m] = M[t + (size_t)c * m];
  if (t < m) a.alpha[t] = (t < nev) ? d[t] : 0.0;
  for (int i = t; i <= m + 1; i += kRsThreads) {
    if (i >= 1 && i < nev) a.beta[i] = e[i - 1];
    else if (i > nev) a.beta[i] = 0.0;
  }
  if (t == 0) {
    a.scal[SC_RCOEF] = M[(m - 1) + (size_t)(nev - 1) * m];
    a.scal[SC_TAU] = (nev < m) ? e[nev - 1] : 0.0;
    state[ST_NCONV] = sh_nconv;
    state[ST_NEV_USE] = nev;
    state[ST_DONE] = 0;
  }
}

size_t restart_scratch_doubles() { return (size_t)4 * kMaxCols * kRsThreads; }

cudaError_t restart_step(const RestartArgs& a, cudaStream_t st) {
  const size_t smem = (size_t)a.m * a.m * sizeof(double) * (a.m <= kRsSmemM ? 5 : 1);
  cudaError_t e = cudaFuncSetAttribute(restart_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  restart_kernel<<<1, kRsThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lg
