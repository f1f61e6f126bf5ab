// lg_adjoint.cu — backward pass of eigsh: gradients of the eigenpairs with
// respect to the stored values of the CSR matrix (implicit differentiation,
// Xie et al. 2020, as the reference's differentiable eigsh).
//
// Reference: python/gpu_eigsh/_cuda_eigsh.cu:183-326 (compute_adjoint_eigsh)
// with src/inner_solve.cuh:69-84 (deflate_against) and :110-200
// (cg_solve_shifted).  For every pair i the reference solves, one after the
// other,  (A - lambda_i I) xi_i = (I - X X^T) gv_i  by CG kept orthogonal to
// span(X) (two Dgemv deflations of Ap and two of r per iteration, four
// blocking reads), copies x_i and xi_i to the host and accumulates
//   grad_vals[p] += (g_i x_i[r] - xi_i[r]) x_i[c]     for entry p = (r, c)
// in a host loop over the nonzeros.
//
// Here the k systems run as ONE block CG on n x ld row-major blocks (ld = k
// rounded up to 8, padding columns kept at zero), each column with its own
// shift, its own scalars and its own convergence test, so every sparse
// product reads the CSR once for all k columns.  One iteration is
//   adj_spmm      AP = A P - P diag(lambda), column dots p.Ap
//   adj_update    alpha = rr / p.Ap;  Xi += alpha P;  R -= alpha AP;  |R|^2
//   adj_gram      D = X^T R                          (FP64 tensor cores)
//   adj_deflate   R -= X D;  |R|^2 = |R|^2 - |D|^2 (X orthonormal);
//                 convergence, beta;  P = R + beta P (FP64 tensor cores)
// Deflating R after every update is the reference's order (deflate Ap,
// update r, deflate r) by linearity: the deflated update of an already
// deflated r equals the deflation of the raw update; p.Ap differs from the
// deflated p.Ap by p.X X^T Ap, which vanishes while p stays orthogonal to X.
// Every reduction ends in a fixed-order sum (last CTA to finish), so results
// are bitwise repeatable.  The gradient is a sampled dense-dense product
// (SDDMM) over the sparsity pattern on the device.
#include "../../include/lanczos_b200.h"
#include "lg_common.cuh"
#include "lg_pool.h"
#include "lg_slq.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

namespace lg {

extern thread_local std::string g_last_error;

namespace adj {

using slq::ColSum;
using slq::kFull;
using slq::kMaxB;
using slq::kRowStride;
using slq::kT;
using slq::kW;
using slq::Lanes;
using slq::Op;
using slq::RowLanes;

constexpr int kDT = 256;                 // threads of the tensor-core kernels
constexpr int kDW = kDT / 32;
constexpr int kGramTile = 32;            // D is reduced in 32 x 32 chunks
constexpr int kGramChunk = kGramTile * kGramTile;
constexpr int kDStride = kMaxB;          // row stride of D (doubles)

// per-column state (doubles unless noted), device
struct State {
  double* lam;        // shifts (the eigenvalues)
  double* rr;         // 2 x kMaxB: |r|^2, double-buffered by iteration parity
  double* tol2;       // (cg_tol |b|)^2 per column
  double* pap;        // ColSum out of adj_spmm (first kMaxB entries)
  double* rraw;       // ColSum out of adj_update
  double* nrm;        // ColSum out of adj_norms
  double* D;          // kMaxB x kDStride
  int* done;          // per column: 0 running, 1 converged, 2 iteration limit, 3 breakdown, 4 zero rhs
  int* iters;         // per column: iterations run
  int* active;        // number of running columns (written by the deflate kernel)
};

__device__ __forceinline__ void dmma(double& c0, double& c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}

// ---------------------------------------------------------------------------
// AP = A P - P diag(lambda); pAp[c] = sum_rows P[row, c] AP[row, c]
// ---------------------------------------------------------------------------
template <int LPR, int NCH>
__global__ void __launch_bounds__(kT, 2)
adj_spmm_kernel(Op op, const double* __restrict__ vals, int k, int ld, const double* __restrict__ P,
                double* __restrict__ AP, State s, ColSum cs) {
  if (*s.active == 0) return;
  using G = RowLanes<double, LPR>;
  constexpr int VEC = G::VEC;
  const G g;
  double lam[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      lam[ch][v] = c < k ? s.lam[c] : 0.0;
    }
  double acc[1][NCH][VEC] = {};
  for (long long wrow = g.first_warp_row(); wrow < op.n; wrow += G::stride()) {
    const long long row = wrow + g.sub;
    const bool valid = row < op.n;
    double y[NCH][VEC], unused[NCH][VEC];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int v = 0; v < VEC; ++v) y[ch][v] = 0.0;
    slq::gather_rows<double, LPR, NCH, false>(op, vals, nullptr, P, ld, k, valid, row, g, y, unused);
    if (!valid) continue;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= k) continue;
      double p[VEC];
      slq::ldvec<double, VEC>(P + row * ld + c0, VEC, p);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        y[ch][v] -= lam[ch][v] * p[v];
        acc[0][ch][v] += p[v] * y[ch][v];
      }
      slq::stvec(AP + row * ld + c0, y[ch], VEC);
    }
  }
  slq::colsum_finish<1, VEC, NCH, LPR>(acc, k, cs);
}

// alpha = rr / pAp (0 for finished columns; a breakdown finishes the column);
// Xi += alpha P; R -= alpha AP; raw |R|^2 per column.
template <int LPR, int NCH>
__global__ void __launch_bounds__(kT, 2)
adj_update_kernel(int n, int k, int ld, int it, const double* __restrict__ P, const double* __restrict__ AP,
                  double* __restrict__ Xi, double* __restrict__ R, State s, ColSum cs) {
  if (*s.active == 0) return;
  __shared__ double s_alpha[kMaxB];
  for (int c = threadIdx.x; c < k; c += kT) {
    double a = 0.0;
    if (s.done[c] == 0) {
      const double pap = s.pap[c];
      if (!(fabs(pap) >= kSafeMin)) {   // breakdown (also NaN): the column stops here
        if (blockIdx.x == 0) {
          s.done[c] = 3;
          s.iters[c] = -(it + 1);
        }
      } else {
        a = s.rr[(it & 1) * kMaxB + c] / pap;
      }
    }
    s_alpha[c] = a;
  }
  __syncthreads();
  using G = RowLanes<double, LPR>;
  constexpr int VEC = G::VEC;
  const G g;
  double al[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      al[ch][v] = c < k ? s_alpha[c] : 0.0;
    }
  double acc[1][NCH][VEC] = {};
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= k) continue;
      double p[VEC], ap[VEC], x[VEC], r[VEC];
      slq::ldvec<double, VEC>(P + row * ld + c0, VEC, p);
      slq::ldvec<double, VEC>(AP + row * ld + c0, VEC, ap);
      slq::ldvec<double, VEC>(Xi + row * ld + c0, VEC, x);
      slq::ldvec<double, VEC>(R + row * ld + c0, VEC, r);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        x[v] += al[ch][v] * p[v];
        r[v] -= al[ch][v] * ap[v];
        acc[0][ch][v] += r[v] * r[v];
      }
      slq::stvec(Xi + row * ld + c0, x, VEC);
      slq::stvec(R + row * ld + c0, r, VEC);
    }
  }
  slq::colsum_finish<1, VEC, NCH, LPR>(acc, k, cs);
}

// Column sums of squares of a block.
template <int LPR, int NCH>
__global__ void __launch_bounds__(kT, 2)
adj_norms_kernel(int n, int k, int ld, const double* __restrict__ B, ColSum cs) {
  using G = RowLanes<double, LPR>;
  constexpr int VEC = G::VEC;
  const G g;
  double acc[1][NCH][VEC] = {};
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= k) continue;
      double b[VEC];
      slq::ldvec<double, VEC>(B + row * ld + c0, VEC, b);
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[0][ch][v] += b[v] * b[v];
    }
  }
  slq::colsum_finish<1, VEC, NCH, LPR>(acc, k, cs);
}

// dst (n x ld, zero padding) = src (n x k, row-major, row stride k), or 0.
__global__ void adj_pad_kernel(int n, int k, int ld, const double* __restrict__ src, double* __restrict__ dst) {
  const long long total = (long long)n * ld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / ld;
    const int c = (int)(i - row * ld);
    dst[i] = (src && c < k) ? src[row * k + c] : 0.0;
  }
}

// ---------------------------------------------------------------------------
// Gram chunk on FP64 tensor cores: part[cta] = X[:, a0:a0+8ta]^T B[:, b0:b0+8tb]
// over this CTA's rows (mma.m8n8k4: K = 4 rows, M = 8 columns of X, N = 8
// columns of B).  Lane (gid, tig) loads X[r0+tig][a0+8ti+gid] and
// B[r0+tig][b0+8tj+gid], exactly its A and B fragments; the warps of a CTA
// are summed in warp order in shared memory.
// ---------------------------------------------------------------------------
// TM: the most 8-column blocks per side (ta, tb <= TM) the instantiation
// holds in registers (a 24-column block of 20 eigenpairs needs 3).
template <int TM>
__global__ void __launch_bounds__(kDT)
adj_gram_kernel(int n, int ld, const double* __restrict__ X, const double* __restrict__ B, int a0, int ta, int b0,
                int tb, double* __restrict__ part, const int* __restrict__ active) {
  if (active && *active == 0) return;
  __shared__ double red[kGramChunk];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  for (int i = t; i < kGramChunk; i += kDT) red[i] = 0.0;
  double acc[TM][TM][2];
#pragma unroll
  for (int ti = 0; ti < TM; ++ti)
#pragma unroll
    for (int tj = 0; tj < TM; ++tj) acc[ti][tj][0] = acc[ti][tj][1] = 0.0;
  const long long step = (long long)gridDim.x * kDW * 4;
  for (long long r0 = ((long long)blockIdx.x * kDW + warp) * 4; r0 < n; r0 += step) {
    const long long row = r0 + tig;
    const bool ok = row < n;
    double xa[TM], bb[TM];
#pragma unroll
    for (int q = 0; q < TM; ++q) {
      xa[q] = (ok && q < ta) ? __ldg(X + row * ld + a0 + 8 * q + gid) : 0.0;
      bb[q] = (ok && q < tb) ? B[row * ld + b0 + 8 * q + gid] : 0.0;
    }
#pragma unroll
    for (int ti = 0; ti < TM; ++ti)
#pragma unroll
      for (int tj = 0; tj < TM; ++tj)
        if (ti < ta && tj < tb) dmma(acc[ti][tj][0], acc[ti][tj][1], xa[ti], bb[tj]);
  }
  __syncthreads();
  for (int w = 0; w < kDW; ++w) {
    if (warp == w) {
#pragma unroll
      for (int ti = 0; ti < TM; ++ti)
#pragma unroll
        for (int tj = 0; tj < TM; ++tj)
          if (ti < ta && tj < tb) {
            double* o = red + (8 * ti + gid) * kGramTile + 8 * tj + 2 * tig;
            o[0] += acc[ti][tj][0];
            o[1] += acc[ti][tj][1];
          }
    }
    __syncthreads();
  }
  for (int i = t; i < kGramChunk; i += kDT) part[(size_t)blockIdx.x * kGramChunk + i] = red[i];
}

// D[a0 + a][b0 + b] = sum over the CTA rows of part, in CTA order: one warp
// per entry (lanes take every 32nd row, then a fixed shuffle tree).
__global__ void adj_gram_reduce_kernel(const double* __restrict__ part, int nparts, int a0, int na, int b0, int nb,
                                       double* __restrict__ D, const int* __restrict__ active) {
  if (active && *active == 0) return;
  const int lane = threadIdx.x & 31;
  const int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (e >= na * nb) return;
  const int a = e / nb, b = e % nb;
  double s = 0.0;
  for (int r = lane; r < nparts; r += 32) s += part[(size_t)r * kGramChunk + a * kGramTile + b];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) D[(size_t)(a0 + a) * kDStride + b0 + b] = s;
}

// ---------------------------------------------------------------------------
// B -= X D on FP64 tensor cores (mma.m8n8k4: M = 8 rows, K = 4 columns of X,
// N = 8 columns of B); D (ld x ld) staged in shared memory.
//   MODE 0 (iteration): B = R; per column the prologue finishes the
//          reductions (|R|^2 = raw - |D col|^2), tests convergence and the
//          iteration limit, and forms beta; then P = R + beta P for the
//          columns still running.
//   MODE 1: B -= X D only (deflation of a right-hand side or of the solution).
// ---------------------------------------------------------------------------
// TBMAX: the most 8-column output blocks (ld / 8) the instantiation holds in
// registers; the narrow blocks of a few eigenpairs keep few accumulators, so
// more CTAs stay resident to stream X, B and P.
template <int MODE, int TBMAX>
__global__ void __launch_bounds__(kDT)
adj_deflate_kernel(int n, int k, int ld, int it, int max_iters, const double* __restrict__ X, double* __restrict__ B,
                   double* __restrict__ P, State s) {
  if (*s.active == 0) return;
  extern __shared__ double sD[];     // ld x ld
  __shared__ double s_beta[kMaxB];
  __shared__ int s_upd[kMaxB];
  __shared__ int s_run;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  for (int i = t; i < ld * ld; i += kDT) sD[i] = s.D[(size_t)(i / ld) * kDStride + (i % ld)];
  if (MODE == 0) {
    if (t == 0) s_run = 0;
    __syncthreads();
    for (int c = t; c < ld; c += kDT) {
      double beta = 0.0;
      int upd = 0;
      if (c < k && s.done[c] == 0) {
        double dn = 0.0;
        for (int a = 0; a < k; ++a) dn += sD[a * ld + c] * sD[a * ld + c];
        const double rr_new = fmax(s.rraw[c] - dn, 0.0);
        if (rr_new < s.tol2[c]) {
          if (blockIdx.x == 0) {
            s.done[c] = 1;
            s.iters[c] = it + 1;
          }
        } else if (it + 1 >= max_iters) {
          if (blockIdx.x == 0) {
            s.done[c] = 2;
            s.iters[c] = -max_iters;
          }
        } else {
          beta = rr_new / s.rr[(it & 1) * kMaxB + c];
          upd = 1;
          if (blockIdx.x == 0) s.rr[((it + 1) & 1) * kMaxB + c] = rr_new;
          atomicAdd(&s_run, 1);
        }
      }
      s_beta[c] = beta;
      s_upd[c] = upd;
    }
  }
  __syncthreads();
  if (MODE == 0 && blockIdx.x == 0 && t == 0) *s.active = s_run;   // read by the next iteration's kernels
  const int TB = ld / 8, KA = ld / 4;
  const long long step = (long long)gridDim.x * kDW * 8;
  for (long long r0 = ((long long)blockIdx.x * kDW + warp) * 8; r0 < n; r0 += step) {
    const long long arow = r0 + gid;
    const bool aok = arow < n;
    double acc[TBMAX][2];
#pragma unroll
    for (int tj = 0; tj < TBMAX; ++tj) acc[tj][0] = acc[tj][1] = 0.0;
    for (int kk = 0; kk < KA; ++kk) {
      const double xa = aok ? __ldg(X + arow * ld + 4 * kk + tig) : 0.0;
#pragma unroll
      for (int tj = 0; tj < TBMAX; ++tj)
        if (tj < TB) dmma(acc[tj][0], acc[tj][1], xa, sD[(4 * kk + tig) * ld + 8 * tj + gid]);
    }
    // lane holds (X D)[r0 + gid][8 tj + 2 tig + {0, 1}]
    if (!aok) continue;
#pragma unroll
    for (int tj = 0; tj < TBMAX; ++tj) {
      if (tj >= TB) break;
      const int c = 8 * tj + 2 * tig;
      double2* bp = reinterpret_cast<double2*>(B + arow * ld + c);
      double2 v = *bp;
      v.x -= acc[tj][0];
      v.y -= acc[tj][1];
      *bp = v;
      if (MODE == 0) {
        double2* pp = reinterpret_cast<double2*>(P + arow * ld + c);
        double2 pv = *pp;
        if (s_upd[c]) pv.x = v.x + s_beta[c] * pv.x;
        if (s_upd[c + 1]) pv.y = v.y + s_beta[c + 1] * pv.y;
        *pp = pv;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// grad[p] = sum_i (g_i X[r, i] - Xi[r, i]) X[c, i] for every stored entry
// p = (r, c) of the CSR: a group of LPR lanes per row broadcasts LPR column
// indices at a time (as gather_rows) and reduces each entry's dot across the
// group.
// ---------------------------------------------------------------------------
template <int LPR, int NCH>
__global__ void __launch_bounds__(kT, 2)
adj_sddmm_kernel(Op op, int k, int ld, const double* __restrict__ X, const double* __restrict__ Xi,
                 const double* __restrict__ g_evals, double* __restrict__ grad) {
  using G = RowLanes<double, LPR>;
  constexpr int VEC = G::VEC;
  const G g;
  double ge[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      ge[ch][v] = (g_evals && c < k) ? g_evals[c] : 0.0;
    }
  const int base = g.lane - g.l;
  for (long long wrow = g.first_warp_row(); wrow < op.n; wrow += G::stride()) {
    const long long row = wrow + g.sub;
    const bool valid = row < op.n;
    double u[NCH][VEC];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      double xr[VEC], xi[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) xr[v] = xi[v] = 0.0;
      if (valid && c0 < k) {
        slq::ldvec<double, VEC>(X + row * ld + c0, VEC, xr);
        slq::ldvec<double, VEC>(Xi + row * ld + c0, VEC, xi);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) u[ch][v] = ge[ch][v] * xr[v] - xi[v];
    }
    const int kb = valid ? __ldg(op.rowptr + row) : 0;
    const int cnt = valid ? __ldg(op.rowptr + row + 1) - kb : 0;
    int mx = cnt;
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) mx = max(mx, __shfl_xor_sync(kFull, mx, o));
    for (int k0 = 0; k0 < mx; k0 += LPR) {
      const int kk = k0 + g.l;
      const int ci = kk < cnt ? __ldg(op.col + kb + kk) : 0;
      const int nb = min(LPR, mx - k0);
      double mine = 0.0;   // this lane's entry k0 + l, after the reductions
      for (int q = 0; q < nb; ++q) {
        const long long c = __shfl_sync(kFull, ci, base + q);
        double d = 0.0;
        if (k0 + q < cnt) {
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            const int c0 = g.col0(ch);
            if (c0 < k) {
              double xc[VEC];
              slq::ldvec<double, VEC>(X + c * ld + c0, VEC, xc);
#pragma unroll
              for (int v = 0; v < VEC; ++v) d += u[ch][v] * xc[v];
            }
          }
        }
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) d += __shfl_xor_sync(kFull, d, o);
        if (g.l == q) mine = d;
      }
      if (kk < cnt) grad[kb + kk] = mine;
    }
  }
}

}  // namespace adj
}  // namespace lg

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace lg {
namespace adj {
namespace {

__global__ void adj_init_kernel(int k, const double* __restrict__ bn2, const double* __restrict__ rr0, double tol,
                                State s) {
  __shared__ int s_run;
  if (threadIdx.x == 0) s_run = 0;
  __syncthreads();
  for (int c = threadIdx.x; c < kMaxB; c += blockDim.x) {
    const bool live = c < k && sqrt(bn2[c]) >= kSafeMin;   // |b| < SAFE_MIN: zero solution, no iterations
    s.done[c] = c < k ? (live ? 0 : 4) : 4;
    s.iters[c] = 0;
    s.rr[c] = c < k ? rr0[c] : 0.0;
    s.tol2[c] = c < k ? tol * tol * bn2[c] : 0.0;
    if (live) atomicAdd(&s_run, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) *s.active = s_run;
}

__global__ void adj_set_kernel(int* p, int v) { *p = v; }

// Structural checks of a device CSR before any kernel gathers through it:
// row_ptr[0] = 0, row_ptr[n] = nnz, row_ptr monotone, 0 <= col < n.
__global__ void adj_check_csr_kernel(int n, long long nnz, const int* __restrict__ rowptr,
                                     const int* __restrict__ col, int* bad) {
  const long long total = std::max((long long)n + 1, nnz);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    if (i <= n) {
      const int rp = rowptr[i];
      if ((i == 0 && rp != 0) || (i == n && rp != nnz) || (i < n && rowptr[i + 1] < rp)) *bad = 1;
    }
    if (i < nnz) {
      const int c = col[i];
      if (c < 0 || c >= n) *bad = 1;
    }
  }
}

int fail(const char* m) {
  g_last_error = std::string("lg_eigsh_adjoint: ") + m;
  return LG_ERR_INVALID;
}

int cuda_fail(cudaError_t e) {
  g_last_error = std::string("lg_eigsh_adjoint: ") + cudaGetErrorString(e);
  return e == cudaErrorMemoryAllocation ? LG_ERR_NOMEM : LG_ERR_CUDA;
}

struct Work {
  int n, k, ld, grid_rl, grid_gram, grid_defl, sms;
  double *X, *P, *AP, *Xi, *R;
  double* part;          // max(grid_rl * kRowStride, grid_gram * kGramChunk)
  ColSum cs_pap, cs_rr, cs_nrm;
  State s;
  double* bn2;           // |rhs|^2 per column (kRowStride)
};

// Lays the workspace out from `base` (nullptr: only sizes it); returns its bytes.
size_t carve(char* base, Work& w) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += (bytes + 255) / 256 * 256;
    return p;
  };
  const size_t blk = sizeof(double) * (size_t)w.n * w.ld;
  w.X = reinterpret_cast<double*>(take(blk));
  w.P = reinterpret_cast<double*>(take(blk));
  w.AP = reinterpret_cast<double*>(take(blk));
  w.Xi = reinterpret_cast<double*>(take(blk));
  w.R = reinterpret_cast<double*>(take(blk));
  w.part = reinterpret_cast<double*>(
      take(sizeof(double) * std::max((size_t)w.grid_rl * kRowStride, (size_t)w.grid_gram * kGramChunk)));
  double* o_pap = reinterpret_cast<double*>(take(sizeof(double) * kRowStride));
  double* o_rr = reinterpret_cast<double*>(take(sizeof(double) * kRowStride));
  double* o_nrm = reinterpret_cast<double*>(take(sizeof(double) * kRowStride));
  w.bn2 = reinterpret_cast<double*>(take(sizeof(double) * kRowStride));
  w.s.lam = reinterpret_cast<double*>(take(sizeof(double) * kMaxB));
  w.s.rr = reinterpret_cast<double*>(take(sizeof(double) * 2 * kMaxB));
  w.s.tol2 = reinterpret_cast<double*>(take(sizeof(double) * kMaxB));
  w.s.D = reinterpret_cast<double*>(take(sizeof(double) * kMaxB * kDStride));
  w.s.done = reinterpret_cast<int*>(take(sizeof(int) * kMaxB));
  w.s.iters = reinterpret_cast<int*>(take(sizeof(int) * kMaxB));
  w.s.active = reinterpret_cast<int*>(take(sizeof(int) * 8));
  unsigned* counters = reinterpret_cast<unsigned*>(take(sizeof(unsigned) * 3));
  w.cs_pap = ColSum{w.part, o_pap, counters + 0};
  w.cs_rr = ColSum{w.part, o_rr, counters + 1};
  w.cs_nrm = ColSum{w.part, o_nrm, counters + 2};
  w.s.pap = o_pap;
  w.s.rraw = o_rr;
  w.s.nrm = o_nrm;
  return off;
}

template <int MODE, int TBMAX>
cudaError_t launch_deflate_tb(const Work& w, int it, int max_iters, double* B, cudaStream_t st) {
  const size_t smem = sizeof(double) * (size_t)w.ld * w.ld;
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = smem_attr_once(attr, (const void*)adj_deflate_kernel<MODE, TBMAX>,
                                 (int)(sizeof(double) * kMaxB * kMaxB));
  if (e != cudaSuccess) return e;
  adj_deflate_kernel<MODE, TBMAX><<<w.grid_defl, kDT, smem, st>>>(w.n, w.k, w.ld, it, max_iters, w.X, B, w.P, w.s);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_deflate(const Work& w, int it, int max_iters, double* B, cudaStream_t st) {
  if (w.ld <= 32) return launch_deflate_tb<MODE, 4>(w, it, max_iters, B, st);
  if (w.ld <= 64) return launch_deflate_tb<MODE, 8>(w, it, max_iters, B, st);
  return launch_deflate_tb<MODE, 16>(w, it, max_iters, B, st);
}

// D = X^T B over every 32 x 32 chunk of (ld x ld).
cudaError_t gram(const Work& w, const double* B, const int* active, cudaStream_t st) {
  for (int a0 = 0; a0 < w.ld; a0 += kGramTile) {
    const int ta = std::min(4, (w.ld - a0) / 8);
    for (int b0 = 0; b0 < w.ld; b0 += kGramTile) {
      const int tb = std::min(4, (w.ld - b0) / 8);
      // one wave of resident CTAs (at most grid_gram, the partial rows' capacity)
      int g = w.grid_gram;
      if (std::max(ta, tb) <= 2) {
        static OccupancyCache occ;
        g = std::min(g, w.sms * resident_blocks_once(occ, (const void*)adj_gram_kernel<2>, kDT, 2));
        adj_gram_kernel<2><<<g, kDT, 0, st>>>(w.n, w.ld, w.X, B, a0, ta, b0, tb, w.part, active);
      } else if (std::max(ta, tb) == 3) {
        static OccupancyCache occ;
        g = std::min(g, w.sms * resident_blocks_once(occ, (const void*)adj_gram_kernel<3>, kDT, 2));
        adj_gram_kernel<3><<<g, kDT, 0, st>>>(w.n, w.ld, w.X, B, a0, ta, b0, tb, w.part, active);
      } else {
        static OccupancyCache occ;
        g = std::min(g, w.sms * resident_blocks_once(occ, (const void*)adj_gram_kernel<4>, kDT, 2));
        adj_gram_kernel<4><<<g, kDT, 0, st>>>(w.n, w.ld, w.X, B, a0, ta, b0, tb, w.part, active);
      }
      const int entries = ta * 8 * tb * 8;
      adj_gram_reduce_kernel<<<(entries * 32 + 255) / 256, 256, 0, st>>>(w.part, g, a0, ta * 8, b0, tb * 8, w.s.D,
                                                                         active);
    }
  }
  return cudaGetLastError();
}

template <int LPR, int NCH>
int run_t(const Op& op, const double* vals, const double* evals, const double* Xin, const double* g_evals,
          const double* g_evecs, double* grad, int max_iters, double tol, int* iters_out, Work& w,
          cudaStream_t st) {
  cudaError_t e;
  const int pad_grid = w.grid_defl;
  adj_pad_kernel<<<pad_grid, 256, 0, st>>>(w.n, w.k, w.ld, Xin, w.X);
  adj_pad_kernel<<<pad_grid, 256, 0, st>>>(w.n, w.k, w.ld, g_evecs, w.R);
  adj_pad_kernel<<<pad_grid, 256, 0, st>>>(w.n, w.k, w.ld, nullptr, w.Xi);
  if ((e = cudaMemsetAsync(w.s.lam, 0, sizeof(double) * kMaxB, st)) != cudaSuccess) return cuda_fail(e);
  if ((e = cudaMemcpyAsync(w.s.lam, evals, sizeof(double) * w.k, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
    return cuda_fail(e);
  if ((e = cudaMemsetAsync(w.cs_pap.counter, 0, 3 * sizeof(unsigned), st)) != cudaSuccess) return cuda_fail(e);
  if ((e = cudaMemsetAsync(w.s.D, 0, sizeof(double) * kMaxB * kDStride, st)) != cudaSuccess) return cuda_fail(e);
  adj_set_kernel<<<1, 1, 0, st>>>(w.s.active, 1);
  // rhs = (I - X X^T) g;  |rhs|;  r0 = (I - X X^T) rhs;  |r0|^2  (the reference
  // deflates the right-hand side, then CG deflates its first residual)
  if ((e = gram(w, w.R, nullptr, st)) != cudaSuccess) return cuda_fail(e);
  if ((e = launch_deflate<1>(w, 0, max_iters, w.R, st)) != cudaSuccess) return cuda_fail(e);
  adj_norms_kernel<LPR, NCH><<<w.grid_rl, kT, 0, st>>>(w.n, w.k, w.ld, w.R, w.cs_nrm);
  if ((e = cudaMemcpyAsync(w.bn2, w.s.nrm, sizeof(double) * kMaxB, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
    return cuda_fail(e);
  if ((e = gram(w, w.R, nullptr, st)) != cudaSuccess) return cuda_fail(e);
  if ((e = launch_deflate<1>(w, 0, max_iters, w.R, st)) != cudaSuccess) return cuda_fail(e);
  adj_norms_kernel<LPR, NCH><<<w.grid_rl, kT, 0, st>>>(w.n, w.k, w.ld, w.R, w.cs_nrm);
  adj_init_kernel<<<1, kMaxB, 0, st>>>(w.k, w.bn2, w.s.nrm, tol, w.s);
  if ((e = cudaMemcpyAsync(w.P, w.R, sizeof(double) * (size_t)w.n * w.ld, cudaMemcpyDeviceToDevice, st)) !=
      cudaSuccess)
    return cuda_fail(e);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e);

  int* h_active = nullptr;
  if ((e = cudaMallocHost(&h_active, sizeof(int))) != cudaSuccess) return cuda_fail(e);
  int it = 0, chunk = 16;
  while (it < max_iters) {
    const int end = std::min(max_iters, it + chunk);
    for (; it < end; ++it) {
      adj_spmm_kernel<LPR, NCH><<<w.grid_rl, kT, 0, st>>>(op, vals, w.k, w.ld, w.P, w.AP, w.s, w.cs_pap);
      adj_update_kernel<LPR, NCH><<<w.grid_rl, kT, 0, st>>>(w.n, w.k, w.ld, it, w.P, w.AP, w.Xi, w.R, w.s,
                                                            w.cs_rr);
      if ((e = gram(w, w.R, w.s.active, st)) != cudaSuccess) break;
      if ((e = launch_deflate<0>(w, it, max_iters, w.R, st)) != cudaSuccess) break;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_active, w.s.active, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess || *h_active == 0) break;
    chunk = std::min(64, chunk * 2);
  }
  cudaFreeHost(h_active);
  if (e != cudaSuccess) return cuda_fail(e);
  // the solution deflated once more (as the reference), then the gradient
  adj_set_kernel<<<1, 1, 0, st>>>(w.s.active, 1);
  if ((e = gram(w, w.Xi, nullptr, st)) != cudaSuccess) return cuda_fail(e);
  if ((e = launch_deflate<1>(w, 0, max_iters, w.Xi, st)) != cudaSuccess) return cuda_fail(e);
  if (op.n > 0)
    adj_sddmm_kernel<LPR, NCH><<<w.grid_rl, kT, 0, st>>>(op, w.k, w.ld, w.X, w.Xi, g_evals, grad);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e);
  if (iters_out) {
    if ((e = cudaMemcpyAsync(iters_out, w.s.iters, sizeof(int) * w.k, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
      return cuda_fail(e);
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_fail(e);
  }
  return LG_OK;
}

}  // namespace
}  // namespace adj
}  // namespace lg

using namespace lg;

extern "C" int lg_eigsh_adjoint(int n, long long nnz, const int* rowptr, const int* col, const double* vals, int k,
                                const double* evals, const double* X, const double* g_evals, const double* g_evecs,
                                double* grad_vals, int cg_max_iters, double cg_tol, int* cg_iters, void* stream) {
  using namespace lg::adj;
  if (n < 1 || nnz < 0 || !rowptr || (nnz > 0 && (!col || !vals || !grad_vals))) return fail("invalid CSR arguments");
  if (nnz > 2147483647ll) return fail("nnz exceeds int32 indexing");
  if (k < 1 || k > kMaxB || k > n) return fail("k must satisfy 1 <= k <= min(n, 128)");
  if (!evals || !X) return fail("null eigenvalues or eigenvectors");
  if (cg_max_iters < 1) return fail("cg_max_iters must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e);
  Work w{};
  w.n = n;
  w.k = k;
  w.ld = (k + 7) / 8 * 8;
  w.grid_rl = 2 * sms;   // the row kernels are built for 2 CTAs of 512 threads per SM
  w.grid_gram = 4 * sms;   // capacity: up to four resident CTAs of the narrow Gram tiles per SM
  w.sms = sms;
  w.grid_defl = 4 * sms;
  void* base = nullptr;
  cudaMemPool_t pool = nullptr;
  if ((e = pool_for(dev, &pool)) != cudaSuccess) return cuda_fail(e);
  if ((e = cudaMallocFromPoolAsync(&base, carve(nullptr, w), pool, st)) != cudaSuccess) return cuda_fail(e);
  carve(static_cast<char*>(base), w);
  {
    int* h_bad = nullptr;
    e = cudaMallocHost(&h_bad, sizeof(int));
    if (e == cudaSuccess) e = cudaMemsetAsync(w.s.active, 0, sizeof(int), st);
    if (e == cudaSuccess) {
      adj_check_csr_kernel<<<4 * sms, 256, 0, st>>>(n, nnz, rowptr, col, w.s.active);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_bad, w.s.active, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    const int bad = (e == cudaSuccess) ? *h_bad : 0;
    if (h_bad) cudaFreeHost(h_bad);
    if (e != cudaSuccess || bad) {
      cudaFreeAsync(base, st);
      return e != cudaSuccess ? cuda_fail(e) : fail("malformed CSR (row_ptr not monotone from 0 to nnz, or a column out of range)");
    }
  }
  const Op op{n, rowptr, col, 0.0};
  int rc;
  if (k <= 32) rc = run_t<16, 1>(op, vals, evals, X, g_evals, g_evecs, grad_vals, cg_max_iters, cg_tol, cg_iters, w, st);
  else if (k <= 64)
    rc = run_t<32, 1>(op, vals, evals, X, g_evals, g_evecs, grad_vals, cg_max_iters, cg_tol, cg_iters, w, st);
  else rc = run_t<32, 2>(op, vals, evals, X, g_evals, g_evecs, grad_vals, cg_max_iters, cg_tol, cg_iters, w, st);
  cudaError_t ef = cudaFreeAsync(base, st);
  if (rc == LG_OK && ef != cudaSuccess) rc = cuda_fail(ef);
  return rc;
}

// Reference-compatible entry point (python/gpu_eigsh/_cuda_eigsh.cu:183-194):
// host arrays, eigenvectors and grad_evecs n x k row-major, returns 0.
extern "C" int compute_adjoint_eigsh(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                                     const double* eigenvalues, const double* eigenvectors, const double* grad_evals,
                                     const double* grad_evecs, double* grad_vals, int cg_max_iters, double cg_tol) {
  if (n < 1 || nnz < 0 || k < 1 || !row_ptr || !eigenvalues || !eigenvectors || (nnz > 0 && (!col_idx || !vals || !grad_vals))) {
    g_last_error = "compute_adjoint_eigsh: invalid arguments";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e != cudaSuccess) return adj::cuda_fail(e);
  const size_t nk = (size_t)n * k;
  char* d = nullptr;
  int *drp = nullptr, *dci = nullptr;
  double *dv = nullptr, *dg = nullptr, *dX = nullptr, *dG = nullptr, *dl = nullptr, *dge = nullptr;
  size_t off = 0;
  auto take = [&](size_t b) { char* p = d ? d + off : nullptr; off += (b + 255) / 256 * 256; return p; };
  auto layout = [&]() {
    off = 0;
    drp = reinterpret_cast<int*>(take(sizeof(int) * ((size_t)n + 1)));
    dci = reinterpret_cast<int*>(take(sizeof(int) * (size_t)std::max(nnz, 1)));
    dv = reinterpret_cast<double*>(take(sizeof(double) * (size_t)std::max(nnz, 1)));
    dg = reinterpret_cast<double*>(take(sizeof(double) * (size_t)std::max(nnz, 1)));
    dX = reinterpret_cast<double*>(take(sizeof(double) * nk));
    dG = grad_evecs ? reinterpret_cast<double*>(take(sizeof(double) * nk)) : nullptr;
    dl = reinterpret_cast<double*>(take(sizeof(double) * k));
    dge = grad_evals ? reinterpret_cast<double*>(take(sizeof(double) * k)) : nullptr;
    return off;
  };
  int rc = LG_OK;
  e = cudaMalloc(&d, layout());
  if (e != cudaSuccess) {
    cudaStreamDestroy(st);
    return adj::cuda_fail(e);
  }
  layout();
  e = cudaMemcpyAsync(drp, row_ptr, sizeof(int) * ((size_t)n + 1), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && nnz > 0) e = cudaMemcpyAsync(dci, col_idx, sizeof(int) * nnz, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && nnz > 0) e = cudaMemcpyAsync(dv, vals, sizeof(double) * nnz, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dX, eigenvectors, sizeof(double) * nk, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && dG) e = cudaMemcpyAsync(dG, grad_evecs, sizeof(double) * nk, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dl, eigenvalues, sizeof(double) * k, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && dge) e = cudaMemcpyAsync(dge, grad_evals, sizeof(double) * k, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) rc = adj::cuda_fail(e);
  if (rc == LG_OK)
    rc = lg_eigsh_adjoint(n, nnz, drp, dci, dv, k, dl, dX, dge, dG, dg, cg_max_iters, cg_tol, nullptr, st);
  if (rc == LG_OK && nnz > 0) {
    e = cudaMemcpyAsync(grad_vals, dg, sizeof(double) * nnz, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = adj::cuda_fail(e);
  }
  cudaStreamSynchronize(st);
  cudaFree(d);
  cudaStreamDestroy(st);
  return rc;
}
