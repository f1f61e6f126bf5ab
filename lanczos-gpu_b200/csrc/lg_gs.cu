// lg_gs.cu — classical Gram-Schmidt passes against the Lanczos basis V.
//
// One Lanczos step j (reference: src/irlm_lanczos.cu:110-148 with
// cgs_orthogonalize / dgks_reorth, src/lanczos_ops.cuh:113-192) is split into
//
//   spmv   : w = A v_j                                    (lg_spmv.cu)
//   pass 1 : h = V^T w,  ||w||^2                          gs_project
//   pass 2 : r1 = w - V h  and  s = V^T r1, ||r1||^2      gs_correct_project
//   pass 3 : r2 = r1 - V s, ||r2||^2, alpha_j = h_j + s_j gs_correct
//
// V is stored ROW-major (n x ldv): a basis row is contiguous, so a warp
// streams rows with its lanes spread over the columns.  In pass 2 the lanes
// hold one row of V in registers, reduce the row dot V[row,:]·h across the
// lanes (shuffles), form r1[row], and immediately accumulate V[row,:]*r1[row]
// into per-lane column sums — the two halves of the pass share one read of
// V.  V is streamed once per pass (three times per step, against four Dgemv
// passes plus copies in the reference); no shared-memory staging, no
// barriers inside the stream.
//
// Lanes per row (LPR) adapt to the live column count: each lane owns two
// adjacent columns per chunk (16-byte loads), a chunk covers 2*LPR columns,
// CH chunks cover up to 2*LPR*CH columns; with fewer columns several rows
// share a warp.  Each CTA owns a contiguous row range and writes one row of
// partial sums; the next kernel reduces those rows in a fixed order in every
// CTA, so results are bitwise repeatable without atomics.
#include "lg_common.cuh"
#include "lg_kernels.cuh"

namespace lg {

constexpr int kGsWarps = kGsThreads / 32;

namespace {

__device__ __forceinline__ double2 ld_stream(const double* p) {
  return __ldcs(reinterpret_cast<const double2*>(p));
}

}  // namespace

// MODE 1: project          (vec = W or R) -> part_out: V^T vec, ||vec||^2
// MODE 2: correct+project  (vec = W)      -> R = vec - V coef ; part_out: V^T R, ||R||^2
// MODE 3: correct          (vec = R)      -> R = vec - V coef ; part_out: ||R||^2
// vec and Rout never alias (MODE 3 reads and writes R through Rout only).
template <int MODE, int LPR, int CH>
__global__ void __launch_bounds__(kGsThreads, 1)
gs_kernel(const double* __restrict__ V, int ldv, int ncols, int n, const double* __restrict__ vec,
          double* __restrict__ Rout, const double* __restrict__ part_in, int nrows_in,
          double* __restrict__ part_out, double* scal, double* alpha, int j, int alpha_mode, int* state) {
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  constexpr int RW = 32 / LPR;     // rows per warp instruction
  // row groups in flight per warp, within the 64-register budget of 1024 threads
  constexpr int U = (MODE == 2) ? 2 : 3;
  constexpr int COLS = 2 * LPR * CH;
  __shared__ double coef[kMaxCols];
  __shared__ double red[kGsThreads];
  __shared__ double wsum[kGsWarps][COLS];
  __shared__ double scr[32];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int sub = lane & (LPR - 1), grp = lane / LPR;

  if (t < kMaxCols) coef[t] = 0.0;
  __syncthreads();
  if (MODE != 1) {
    double sc;
    reduce_partials(part_in, nrows_in, ncols, coef, &sc, red);
    if (blockIdx.x == 0 && t == 0) {
      if (MODE == 2) {
        scal[SC_WN2] = sc;
        scal[SC_HJ] = coef[ncols - 1];
      } else {
        scal[SC_R1N2] = sc;
        if (alpha_mode == 1) alpha[j] = scal[SC_HJ] + coef[j];
        else if (alpha_mode == 2) alpha[j] += coef[j];
      }
    }
  }

  double2 cf[CH];
  bool live[CH], pair[CH];   // pair: the second column of the lane's 16-byte chunk is live too
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int c0 = ch * 2 * LPR + 2 * sub;
    live[ch] = c0 < ncols;
    pair[ch] = c0 + 1 < ncols;
    cf[ch] = make_double2(coef[c0], coef[c0 + 1]);
  }
  double2 acc[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) acc[ch] = make_double2(0.0, 0.0);
  double nrm = 0.0;

  const long long rb = (long long)n * blockIdx.x / gridDim.x;
  const long long re = (long long)n * (blockIdx.x + 1) / gridDim.x;
  const long long step = (long long)kGsWarps * RW;

  // the loop bound is warp-uniform (row groups only differ by grp < RW)
  for (long long w0 = rb + (long long)warp * RW; w0 < re; w0 += step * U) {
    const long long r0 = w0 + grp;
    double2 v[U][CH];
    double x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long r = r0 + u * step;
      const bool ok = r < re;
      const double* row = V + r * ldv;
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) {
        v[u][ch] = (ok && live[ch]) ? ld_stream(row + ch * 2 * LPR + 2 * sub) : make_double2(0.0, 0.0);
        if (!pair[ch]) v[u][ch].y = 0.0;   // padding column: never let its contents in
      }
      x[u] = ok ? (MODE == 3 ? Rout[r] : vec[r]) : 0.0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long r = r0 + u * step;
      const bool ok = r < re;
      if (MODE == 1) {
#pragma unroll
        for (int ch = 0; ch < CH; ++ch) {
          acc[ch].x += v[u][ch].x * x[u];
          acc[ch].y += v[u][ch].y * x[u];
        }
        if (ok && sub == 0) nrm += x[u] * x[u];
      } else {
        double d = 0.0;
#pragma unroll
        for (int ch = 0; ch < CH; ++ch) d += v[u][ch].x * cf[ch].x + v[u][ch].y * cf[ch].y;
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const double y = x[u] - d;
        if (ok && sub == 0) {
          Rout[r] = y;
          nrm += y * y;
        }
        if (MODE == 2) {
#pragma unroll
          for (int ch = 0; ch < CH; ++ch) {
            acc[ch].x += v[u][ch].x * y;
            acc[ch].y += v[u][ch].y * y;
          }
        }
      }
    }
  }

  double* prow = part_out + (size_t)blockIdx.x * kPartStride;
  if (MODE != 3) {
    // reduce the row groups of the warp, then the warps of the CTA
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
#pragma unroll
      for (int o = 16; o >= LPR; o >>= 1) {
        acc[ch].x += __shfl_xor_sync(0xffffffffu, acc[ch].x, o);
        acc[ch].y += __shfl_xor_sync(0xffffffffu, acc[ch].y, o);
      }
      if (grp == 0) {
        const int c0 = ch * 2 * LPR + 2 * sub;
        wsum[warp][c0] = acc[ch].x;
        wsum[warp][c0 + 1] = acc[ch].y;
      }
    }
    __syncthreads();
    if (t < ncols) {
      double s = 0.0;
      for (int w = 0; w < kGsWarps; ++w) s += wsum[w][t];
      prow[t] = s;
    }
  }
  const double tot = block_sum(nrm, scr);
  if (t == 0) prow[kPartScalar] = tot;
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
GsPlan gs_plan(int n, int ncols, int grid) {
  GsPlan p;
  p.grid = grid;
  // four columns per lane (two 16-byte chunks): the row-dot reduction is
  // log2(lpr) shuffles shared by 32/lpr rows
  p.ch = 2;
  if (ncols <= 16) p.lpr = 4;
  else if (ncols <= 32) p.lpr = 8;
  else if (ncols <= 64) p.lpr = 16;
  else p.lpr = 32;
  const long long rows_per_cta = (long long)(n + grid - 1) / grid;
  if (rows_per_cta < 1) p.grid = n;
  return p;
}

template <int MODE>
static cudaError_t launch_mode(const GsPlan& p, cudaStream_t st, const double* V, int ldv, int ncols, int n,
                               const double* vec, double* Rout, const double* part_in, int nrows_in,
                               double* part_out, double* scal, double* alpha, int j, int alpha_mode, int* state) {
#define LG_GS(LP, C)                                                                                          \
  gs_kernel<MODE, LP, C><<<p.grid, kGsThreads, 0, st>>>(V, ldv, ncols, n, vec, Rout, part_in, nrows_in,      \
                                                        part_out, scal, alpha, j, alpha_mode, state)
  if (p.lpr == 4) LG_GS(4, 2);
  else if (p.lpr == 8) LG_GS(8, 2);
  else if (p.lpr == 16) LG_GS(16, 2);
  else LG_GS(32, 2);
#undef LG_GS
  return cudaGetLastError();
}

cudaError_t gs_project(const GsPlan& p, cudaStream_t st, const double* V, int ldv, int ncols, int n,
                       const double* vec, double* part_out, int* state) {
  return launch_mode<1>(p, st, V, ldv, ncols, n, vec, nullptr, nullptr, 0, part_out, nullptr, nullptr, 0, 0,
                        state);
}

cudaError_t gs_correct_project(const GsPlan& p, cudaStream_t st, const double* V, int ldv, int ncols, int n,
                               const double* W, double* R, const double* part_in, int nrows_in,
                               double* part_out, double* scal, int* state) {
  return launch_mode<2>(p, st, V, ldv, ncols, n, W, R, part_in, nrows_in, part_out, scal, nullptr, 0, 0, state);
}

cudaError_t gs_correct(const GsPlan& p, cudaStream_t st, const double* V, int ldv, int ncols, int n, double* R,
                       const double* part_in, int nrows_in, double* part_out, double* scal, double* alpha,
                       int j, int alpha_mode, int* state) {
  return launch_mode<3>(p, st, V, ldv, ncols, n, nullptr, R, part_in, nrows_in, part_out, scal, alpha, j,
                        alpha_mode, state);
}

}  // namespace lg
