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
// V has the layout L (lg_kernels.cuh): the solver keeps it in panels of 8
// columns, the caller of lg_cgs2_orthogonalize row-major; either way a lane
// loads 16-byte chunks of two adjacent columns of a row, and a warp streams
// rows with its lanes spread over the columns.  In pass 2 the lanes
// hold one row of V in registers, reduce the row dot V[row,:]·h across the
// lanes (shuffles), form r1[row], and immediately accumulate V[row,:]*r1[row]
// into per-lane column sums — the two halves of the pass share one read of
// V.  V is streamed once per pass (three times per step, against four Dgemv
// passes plus copies in the reference), with no barriers inside the stream:
// pass 1 from plain loads (three row groups in flight per warp), passes 2 and
// 3 through a per-warp ring of asynchronous copies (gs_async_kernel).
//
// Lanes per row (LPR) adapt to the live column count: each lane owns two
// adjacent columns per chunk (16-byte loads), a chunk covers 2*LPR columns,
// CH chunks cover up to 2*LPR*CH columns; with fewer columns several rows
// share a warp.  Each CTA owns a contiguous row range and writes one row of
// partial sums; the next kernel reduces those rows in a fixed order in every
// CTA, so results are bitwise repeatable without atomics.
#include "lg_common.cuh"
#include "lg_kernels.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

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
gs_kernel(const double* __restrict__ V, VLayout L, int ncols, int n, const double* __restrict__ vec,
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
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) {
        v[u][ch] = (ok && live[ch]) ? ld_stream(V + vidx(L, r, ch * 2 * LPR + 2 * sub)) : make_double2(0.0, 0.0);
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
// The same three passes with the V stream staged through shared memory by
// asynchronous copies (cp.async, 16 bytes per lane, completion per thread).
// A plain-load loop keeps at most U row groups of V in flight per warp (the
// loads must land in registers); here every warp keeps kGsStages - 1 row
// groups in flight in its private ring of shared memory while it computes on
// the oldest one, with no register cost and no block-wide barrier: each lane
// reads back the 16-byte chunks it copied itself; the row's entry of vec / R
// is copied by the first lane of the row group and read by the group after a
// __syncwarp.  Everything else (lane layout, sums, outputs) is gs_kernel's.
// ---------------------------------------------------------------------------
constexpr int kGsStages = 4;
constexpr int kGsStageDoubles = 32 * 2 * 2 + 8;   // 32 lanes x 2 chunks x 2 doubles, 8 row entries

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int bytes) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, int bytes) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(sa), "l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

size_t gs_async_smem() { return sizeof(double) * (size_t)kGsWarps * kGsStages * kGsStageDoubles; }

template <int MODE, int LPR>
__global__ void __launch_bounds__(kGsThreads, 1)
gs_async_kernel(const double* __restrict__ V, VLayout L, int ncols, int n, const double* __restrict__ vec,
                double* __restrict__ Rout, const double* __restrict__ part_in, int nrows_in,
                double* __restrict__ part_out, double* scal, double* alpha, int j, int alpha_mode, int* state) {
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  constexpr int CH = 2;
  constexpr int RW = 32 / LPR;     // rows per row group (one per lane group)
  constexpr int COLS = 2 * LPR * CH;
  static_assert(RW <= 8, "row entries per stage");
  extern __shared__ __align__(16) double gs_ring[];
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
  bool live[CH], pair[CH];
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
  const long long wfirst = rb + (long long)warp * RW;
  const long long ngroups = wfirst < re ? (re - wfirst + step - 1) / step : 0;   // warp-uniform
  double* ring = gs_ring + (size_t)warp * kGsStages * kGsStageDoubles;
  const double* xsrc = MODE == 3 ? Rout : vec;

  auto issue = [&](long long gi) {
    double* st = ring + (int)(gi % kGsStages) * kGsStageDoubles;
    const long long r = wfirst + gi * step + grp;
    const bool ok = gi < ngroups && r < re;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      const bool go = ok && live[ch];
      cp_async16(st + (ch * 32 + lane) * 2, go ? V + vidx(L, r, ch * 2 * LPR + 2 * sub) : V, go ? 16 : 0);
    }
    if (sub == 0) cp_async8(st + 128 + grp, ok ? xsrc + r : xsrc, ok ? 8 : 0);
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < kGsStages - 1; ++s) issue(s);
  for (long long gi = 0; gi < ngroups; ++gi) {
    __syncwarp();                    // every lane is done with the stage about to be refilled
    issue(gi + kGsStages - 1);
    cp_async_wait<kGsStages - 1>();  // this lane's copies of group gi have landed
    __syncwarp();                    // ... and those of the other lanes (row entries)
    const double* st = ring + (int)(gi % kGsStages) * kGsStageDoubles;
    const long long r = wfirst + gi * step + grp;
    const bool ok = r < re;
    double2 v[CH];
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      v[ch] = *reinterpret_cast<const double2*>(st + (ch * 32 + lane) * 2);
      if (!pair[ch]) v[ch].y = 0.0;   // padding column: never let its contents in
    }
    const double x = st[128 + grp];
    if (MODE == 1) {
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) {
        acc[ch].x += v[ch].x * x;
        acc[ch].y += v[ch].y * x;
      }
      if (ok && sub == 0) nrm += x * x;
    } else {
      double d = 0.0;
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) d += v[ch].x * cf[ch].x + v[ch].y * cf[ch].y;
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const double y = x - d;
      if (ok && sub == 0) {
        Rout[r] = y;
        nrm += y * y;
      }
      if (MODE == 2) {
#pragma unroll
        for (int ch = 0; ch < CH; ++ch) {
          acc[ch].x += v[ch].x * y;
          acc[ch].y += v[ch].y * y;
        }
      }
    }
  }
  cp_async_wait<0>();

  double* prow = part_out + (size_t)blockIdx.x * kPartStride;
  if (MODE != 3) {
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
// Lag steps: the second Gram-Schmidt pass of step j-1 delayed into step j
// (the delayed reorthogonalisation of low-synchronisation CGS2, Swirydowicz,
// Langou, Ananthan, Yang, Thomas 2020; Bielich et al. 2022), two streams of V
// per Lanczos step instead of three.
//
// Entering step j the basis has j finished columns and R holds u, the
// residual of step j-1 after ONE pass (u = r1).  With rho = ||u||:
//   spmv (BETA_LAG)   z = A u / rho
//   gs_lag_project    s = V^T u, t = V^T z, u^T z, ||u||^2     (one read of V)
//   gs_lag_correct    beta_j = sqrt(||u||^2 - ||s||^2)         (the norm of the
//                       twice-orthogonalised residual u - V s)
//                     v_j = (u - V s) / beta_j                 -> V[:, j]
//                     alpha_{j-1} += s_{j-1}                   (its second-pass term)
//                     v_j^T z = (u^T z - s.t) / beta_j
//                     r1 = (rho / beta_j) (z - V t - (v_j^T z) v_j)  -> R
//                     alpha_j = rho (v_j^T z) / beta_j - s_{j-1}     (first pass)
// Since A v_j = (rho z - A V s) / beta_j and, by the Lanczos relation,
// A V s = V T s + beta_j s_{j-1} v_j, the projections of A v_j are
// V^T A v_j = (rho t - T s) / beta_j and v_j^T A v_j = alpha_j above; r1 is
// then exactly (rho / beta_j)(z - V t - (v_j^T z) v_j): the T s terms cancel.
// Only the alpha update uses the relation, through a term of the size of s
// (a rounding-level quantity), so the basis, alpha and beta agree with the
// in-step CGS2 to rounding.  The DGKS test of the reference (rnorm after the
// second pass <= ||r1|| / sqrt(2)) becomes beta_j^2 <= ||u||^2 / 2 and ends the
// step with STATUS_PASS3_LAG; the breakdown test is the reference's, on beta_j.
// ---------------------------------------------------------------------------
// Layout: 16 warps per CTA (512 threads, so the coefficient and chunk
// registers of four 16-byte chunks per lane fit without spills), LPR lanes
// per basis row, each lane holding four 16-byte chunks (8 columns), so a
// warp iteration covers 32/LPR rows: LPR = 4, 8, 16 for up to 32, 64, 128
// live columns, 8, 4, 2 rows per iteration.  A per-warp cp.async ring stages
// the V chunks and the rows' entries of u and z.
constexpr int kLagWarps = 16;
constexpr int kLagThreads = kLagWarps * 32;
constexpr int kLagCH = 4;
constexpr int kLagStageDoubles = 32 * kLagCH * 2 + 16;   // V chunks, 8 entries of u, 8 of z

size_t gs_lag_smem() { return sizeof(double) * (size_t)kLagWarps * kGsStages * kLagStageDoubles; }

template <int LPR, int CL>
__global__ void __launch_bounds__(kLagThreads, 1)
gs_lag_project_kernel(const double* __restrict__ V, VLayout L, int ncols, int n, const double* __restrict__ U,
                      const double* __restrict__ Z, double* __restrict__ partS, double* __restrict__ partT,
                      int* state) {
  griddep_wait();   // Z comes from the sparse product just before
  griddep_launch_dependents();
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  constexpr int CH = kLagCH;
  constexpr int RW = 32 / LPR;
  constexpr int COLS = 2 * LPR * CH;
  static_assert(RW <= 8, "row entries per stage");
  extern __shared__ __align__(16) double gs_ring[];
  __shared__ double wsum[kLagWarps][COLS];
  __shared__ double scr[32];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int sub = lane & (LPR - 1), grp = lane / LPR;
  bool live[CH], pair[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int c0 = ch * 2 * LPR + 2 * sub;
    live[ch] = c0 < ncols;
    pair[ch] = c0 + 1 < ncols;
  }
  double2 as[CH], at[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    as[ch] = make_double2(0.0, 0.0);
    at[ch] = make_double2(0.0, 0.0);
  }
  double uz = 0.0, uu = 0.0, zz = 0.0;

  const int rb = (int)((long long)n * blockIdx.x / gridDim.x);
  const int re = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
  constexpr int step = kLagWarps * RW;
  const int wfirst = rb + warp * RW;
  const int ngroups = wfirst < re ? (re - wfirst + step - 1) / step : 0;   // warp-uniform
  double* ring = gs_ring + (size_t)warp * kGsStages * kLagStageDoubles;

  auto issue = [&](int gi) {
    double* st = ring + (gi % kGsStages) * kLagStageDoubles;
    const int r = wfirst + gi * step + grp;
    const bool ok = gi < ngroups && r < re;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      const bool go = ok && live[ch];
      cp_async16(st + (ch * 32 + lane) * 2, go ? V + vidx(L, r, ch * 2 * LPR + 2 * sub) : V, go ? 16 : 0);
    }
    if (sub == 0) {
      cp_async8(st + 32 * CH * 2 + grp, ok ? U + r : U, ok ? 8 : 0);
      cp_async8(st + 32 * CH * 2 + 8 + grp, ok ? Z + r : Z, ok ? 8 : 0);
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < kGsStages - 1; ++s) issue(s);
  for (int gi = 0; gi < ngroups; ++gi) {
    __syncwarp();
    issue(gi + kGsStages - 1);
    cp_async_wait<kGsStages - 1>();
    __syncwarp();
    const double* st = ring + (gi % kGsStages) * kLagStageDoubles;
    const int r = wfirst + gi * step + grp;
    const bool ok = r < re;
    const double xu = st[32 * CH * 2 + grp], xz = st[32 * CH * 2 + 8 + grp];
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      double2 v = *reinterpret_cast<const double2*>(st + (ch * 32 + lane) * 2);
      if (!pair[ch]) v.y = 0.0;
      as[ch].x += v.x * xu;
      as[ch].y += v.y * xu;
      at[ch].x += v.x * xz;
      at[ch].y += v.y * xz;
    }
    if (ok && sub == 0) {
      uz += xu * xz;
      uu += xu * xu;
      zz += xz * xz;
    }
  }
  cp_async_wait<0>();

  // column sums into this CTA's rows: s through wsum first, then t
  __shared__ double rowS[kPartStride], rowT[kPartStride];
  for (int pass = 0; pass < 2; ++pass) {
    double2* acc = pass == 0 ? as : at;
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
    double* row = pass == 0 ? rowS : rowT;
    if (t < ncols) {
      double sum = 0.0;
      for (int w = 0; w < kLagWarps; ++w) sum += wsum[w][t];
      row[t] = sum;
    }
    __syncthreads();
  }
  const double tuz = block_sum(uz, scr);
  const double tuu = block_sum(uu, scr);
  const double tzz = block_sum(zz, scr);
  if (t == 0) {
    rowS[ncols] = tuu;
    rowS[kPartScalar] = tuz;
    rowT[kPartScalar] = tzz;
  }
  if (CL == 1) {
    __syncthreads();
    double* ps = partS + (size_t)blockIdx.x * kPartStride;
    double* pt = partT + (size_t)blockIdx.x * kPartStride;
    if (t <= ncols) ps[t] = rowS[t];
    if (t < ncols) pt[t] = rowT[t];
    if (t == 0) {
      ps[kPartScalar] = tuz;
      pt[kPartScalar] = tzz;
    }
  } else {
    // the CL CTAs of a cluster add their rows (ranks in order, through
    // distributed shared memory) into one row: the correction reduces CL
    // times fewer rows in its prologue
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0) {
      const int slot = t < kPartStride ? t : t - kPartStride;   // threads [0, 136): S, [136, 272): T
      const bool isT = t >= kPartStride;
      const bool used = t < 2 * kPartStride &&
                        (isT ? (slot < ncols || slot == kPartScalar) : (slot <= ncols || slot == kPartScalar));
      if (used) {
        double sum = 0.0;
#pragma unroll
        for (int q = 0; q < CL; ++q) sum += cluster.map_shared_rank(isT ? rowT : rowS, q)[slot];
        (isT ? partT : partS)[(size_t)(blockIdx.x / CL) * kPartStride + slot] = sum;
      }
    }
    cluster.sync();   // the other CTAs' rows stay alive until they are read
  }
}

template <int LPR>
__global__ void __launch_bounds__(kLagThreads, 1)
gs_lag_correct_kernel(double* V, VLayout L, int ncols, int n, double* R, const double* __restrict__ Z,
                      const double* __restrict__ partS, const double* __restrict__ partT, int nrows_in,
                      double* __restrict__ part_out, double* scal, double* alpha, double* beta, int* state) {
  constexpr int CH = kLagCH;
  constexpr int RW = 32 / LPR;
  static_assert(RW <= 8, "row entries per stage");
  extern __shared__ __align__(16) double gs_ring[];
  __shared__ double cs[kMaxCols + 1], ct[kMaxCols + 1];
  __shared__ double wred[2][8][kMaxCols + 2];
  __shared__ double scr[32];
  __shared__ double sh_b1, sh_b2, sh_rb, sh_vjz, sh_uz, sh_zz;
  __shared__ int sh_stop;

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int sub = lane & (LPR - 1), grp = lane / LPR;
  const int j = ncols;   // the column this step finishes

  bool live[CH], pair[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int c0 = ch * 2 * LPR + 2 * sub;
    live[ch] = c0 < ncols;
    pair[ch] = c0 + 1 < ncols;
  }
  const int rb0 = (int)((long long)n * blockIdx.x / gridDim.x);
  const int re = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
  constexpr int step = kLagWarps * RW;
  const int wfirst = rb0 + warp * RW;
  const int ngroups = wfirst < re ? (re - wfirst + step - 1) / step : 0;   // warp-uniform
  double* ring = gs_ring + (size_t)warp * kGsStages * kLagStageDoubles;
  auto issue = [&](int gi) {
    double* st = ring + (gi % kGsStages) * kLagStageDoubles;
    const int r = gi < ngroups ? wfirst + (ngroups - 1 - gi) * step + grp : re;
    const bool ok = r < re;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      const bool go = ok && live[ch];
      cp_async16(st + (ch * 32 + lane) * 2, go ? V + vidx(L, r, ch * 2 * LPR + 2 * sub) : V, go ? 16 : 0);
    }
    if (sub == 0) {
      cp_async8(st + 32 * CH * 2 + grp, ok ? R + r : R, ok ? 8 : 0);
      cp_async8(st + 32 * CH * 2 + 8 + grp, ok ? Z + r : Z, ok ? 8 : 0);
    }
    cp_async_commit();
  };
  // The first row groups are in flight while the partial sums are reduced.
  // V's live columns, u and z were final before the projection started, so
  // these copies may run before this kernel waits for the projection; its
  // partial sums and the state word are read after the wait.
#pragma unroll
  for (int s = 0; s < kGsStages - 1; ++s) issue(s);
  griddep_wait();
  griddep_launch_dependents();
  if (state[ST_STATUS] != STATUS_RUNNING) {
    cp_async_wait<0>();   // no copy may still target shared memory when the CTA exits
    return;
  }

  // partial-sum tables: threads [0, 256) table S (columns 0..j, scalar u^T z),
  // [256, 512) table T (columns 0..j-1, scalar ||z||^2); warp w of a half sums
  // rows w, w + 8, ... in order (all loads of a lane independent), then the
  // eight warps in order
  {
    const int half = t >> 8, w8 = (t >> 5) & 7;
    const double* part = half == 0 ? partS : partT;
    const int nc = half == 0 ? ncols + 1 : ncols;   // columns, then the scalar slot as entry nc
    double acc[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
    int colx[5];
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = lane + 32 * q;
      colx[q] = i < nc ? i : (i == nc ? kPartScalar : -1);
    }
    int r = w8;
    for (; r + 24 < nrows_in; r += 32) {
#pragma unroll
      for (int q = 0; q < 5; ++q) {
        if (colx[q] < 0) continue;
        const double* pc = part + colx[q];
        const double a0 = __ldcg(pc + (size_t)r * kPartStride), a1 = __ldcg(pc + (size_t)(r + 8) * kPartStride);
        const double a2 = __ldcg(pc + (size_t)(r + 16) * kPartStride), a3 = __ldcg(pc + (size_t)(r + 24) * kPartStride);
        acc[q] += a0;
        acc[q] += a1;
        acc[q] += a2;
        acc[q] += a3;
      }
    }
    for (; r < nrows_in; r += 8) {
#pragma unroll
      for (int q = 0; q < 5; ++q)
        if (colx[q] >= 0) acc[q] += __ldcg(part + (size_t)r * kPartStride + colx[q]);
    }
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int i = lane + 32 * q;
      if (i <= nc) wred[half][w8][i] = acc[q];
    }
  }
  __syncthreads();
  if (t < 2 * (kMaxCols + 2)) {
    const int half = t >= kMaxCols + 2 ? 1 : 0, i = t - half * (kMaxCols + 2);
    const int nc = half == 0 ? ncols + 1 : ncols;
    if (i <= nc) {
      double s = 0.0;
#pragma unroll
      for (int w = 0; w < 8; ++w) s += wred[half][w][i];
      if (i < nc) (half == 0 ? cs : ct)[i] = s;
      else if (half == 0) sh_uz = s;
      else sh_zz = s;
    }
  }
  __syncthreads();
  if (t < 32) {
    double ss = 0.0, st = 0.0;
    for (int i = t; i < ncols; i += 32) {
      ss += cs[i] * cs[i];
      st += cs[i] * ct[i];
    }
    ss = warp_sum(ss);
    st = warp_sum(st);
    const double uu = cs[j];
    const double aprev = scal[SC_ALPHA_PREV] + cs[j - 1];
    const double btol = breakdown_tol_warp(alpha, beta, j - 1, true, aprev);
    if (t == 0) {
      const double uz = sh_uz;
      const double b2 = uu - ss;
      const double b = b2 > 0.0 ? sqrt(b2) : 0.0;
      int stop = STATUS_RUNNING;
      if (!(b2 > 0.5 * uu)) stop = STATUS_PASS3_LAG;
      else if (b < btol) stop = STATUS_BREAKDOWN;
      double s1 = 1.0, s2 = 1.0;
      safe_inv(b, s1, s2);
      const double rho = scal[SC_BETA_NEXT];
      const double vjz = ((uz - st) * s1) * s2;
      sh_b1 = s1;
      sh_b2 = s2;
      sh_rb = ((rho * s1) * s2);
      sh_vjz = vjz;
      sh_stop = stop;
      if (blockIdx.x == 0) {
        if (stop != STATUS_RUNNING) {
          state[ST_STEP] = j - 1;
          state[ST_STATUS] = stop;
        } else {
          alpha[j - 1] = aprev;
          beta[j] = b;
          alpha[j] = ((rho * vjz) * s1) * s2 - cs[j - 1];
        }
      }
    }
  }
  __syncthreads();
  if (sh_stop != STATUS_RUNNING) {
    cp_async_wait<0>();   // no copy may still target shared memory when the CTA exits
    return;
  }
  const double b1 = sh_b1, b2s = sh_b2, rb = sh_rb, vjz = sh_vjz;

  double2 c1[CH], c2[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    const int c0 = ch * 2 * LPR + 2 * sub;
    c1[ch] = make_double2(c0 < ncols ? cs[c0] : 0.0, c0 + 1 < ncols ? cs[c0 + 1] : 0.0);
    c2[ch] = make_double2(c0 < ncols ? ct[c0] : 0.0, c0 + 1 < ncols ? ct[c0 + 1] : 0.0);
  }
  double nrm = 0.0;

  for (int gi = 0; gi < ngroups; ++gi) {
    __syncwarp();
    issue(gi + kGsStages - 1);
    cp_async_wait<kGsStages - 1>();
    __syncwarp();
    const double* st = ring + (gi % kGsStages) * kLagStageDoubles;
    const int r = wfirst + (ngroups - 1 - gi) * step + grp;
    double d1 = 0.0, d2 = 0.0;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      double2 v = *reinterpret_cast<const double2*>(st + (ch * 32 + lane) * 2);
      if (!pair[ch]) v.y = 0.0;
      d1 += v.x * c1[ch].x + v.y * c1[ch].y;
      d2 += v.x * c2[ch].x + v.y * c2[ch].y;
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) {
      d1 += __shfl_xor_sync(0xffffffffu, d1, o);
      d2 += __shfl_xor_sync(0xffffffffu, d2, o);
    }
    if (r < re && sub == 0) {
      const double xu = st[32 * CH * 2 + grp], xz = st[32 * CH * 2 + 8 + grp];
      const double vj = ((xu - d1) * b1) * b2s;
      const double r1 = rb * (xz - d2 - vjz * vj);
      V[vidx(L, r, j)] = vj;
      R[r] = r1;
      nrm += r1 * r1;
    }
  }
  cp_async_wait<0>();
  const double tot = block_sum(nrm, scr);
  if (t == 0) part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = tot;
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

// Passes 2 and 3 stream V through the cp.async ring (gs_async_kernel): measured
// 7 % and 5 % faster than the register loop on configuration 1; pass 1 keeps
// the register loop with three row groups in flight (4 % faster there).
constexpr bool kGsAsync2 = true, kGsAsync3 = true, kGsAsync1 = false;

template <int MODE>
static cudaError_t launch_mode(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                               const double* vec, double* Rout, const double* part_in, int nrows_in,
                               double* part_out, double* scal, double* alpha, int j, int alpha_mode, int* state) {
  if ((MODE == 1 && kGsAsync1) || (MODE == 2 && kGsAsync2) || (MODE == 3 && kGsAsync3)) {
#define LG_GSA(LP)                                                                                              \
  do {                                                                                                          \
    static std::atomic<unsigned long long> attr{0};                                                             \
    cudaError_t e = smem_attr_once(attr, (const void*)gs_async_kernel<MODE, LP>, (int)gs_async_smem());         \
    if (e != cudaSuccess) return e;                                                                             \
    gs_async_kernel<MODE, LP><<<p.grid, kGsThreads, gs_async_smem(), st>>>(V, L, ncols, n, vec, Rout, part_in,    \
                                                                          nrows_in, part_out, scal, alpha, j,   \
                                                                          alpha_mode, state);                   \
  } while (0)
    if (p.lpr == 4) LG_GSA(4);
    else if (p.lpr == 8) LG_GSA(8);
    else if (p.lpr == 16) LG_GSA(16);
    else LG_GSA(32);
#undef LG_GSA
    return cudaGetLastError();
  }
#define LG_GS(LP, C)                                                                                          \
  gs_kernel<MODE, LP, C><<<p.grid, kGsThreads, 0, st>>>(V, L, ncols, n, vec, Rout, part_in, nrows_in,        \
                                                        part_out, scal, alpha, j, alpha_mode, state)
  if (p.lpr == 4) LG_GS(4, 2);
  else if (p.lpr == 8) LG_GS(8, 2);
  else if (p.lpr == 16) LG_GS(16, 2);
  else LG_GS(32, 2);
#undef LG_GS
  return cudaGetLastError();
}

cudaError_t gs_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                       const double* vec, double* part_out, int* state) {
  return launch_mode<1>(p, st, V, L, ncols, n, vec, nullptr, nullptr, 0, part_out, nullptr, nullptr, 0, 0,
                        state);
}

cudaError_t gs_correct_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                               const double* W, double* R, const double* part_in, int nrows_in,
                               double* part_out, double* scal, int* state) {
  return launch_mode<2>(p, st, V, L, ncols, n, W, R, part_in, nrows_in, part_out, scal, nullptr, 0, 0, state);
}

cudaError_t gs_correct(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n, double* R,
                       const double* part_in, int nrows_in, double* part_out, double* scal, double* alpha,
                       int j, int alpha_mode, int* state) {
  return launch_mode<3>(p, st, V, L, ncols, n, nullptr, R, part_in, nrows_in, part_out, scal, alpha, j,
                        alpha_mode, state);
}


// Cluster size of the projection: the largest of 4 and 2 that divides the grid
// and lets every cluster be resident at once (GPCs whose SM count is not a
// multiple of the cluster size leave SMs out, and a second wave would cost
// more than the shorter prologue saves), else 1.  Decided once per device
// and grid from the occupancy query.
template <int CL>
static bool cluster_fits(int grid) {
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = smem_attr_once(attr, (const void*)gs_lag_project_kernel<8, CL>, (int)gs_lag_smem());
  int active = 0;
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLagThreads);
    cfg.dynamicSmemBytes = gs_lag_smem();
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&active, (const void*)gs_lag_project_kernel<8, CL>, &cfg);
  }
  if (e != cudaSuccess) cudaGetLastError();
  return e == cudaSuccess && (long long)active * CL >= grid;
}

static int lag_cluster(int grid) {
  static std::atomic<long long> cache[64];   // per device: (grid << 8) | cluster, 0 unknown
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  const long long c = cache[dev].load();
  if (c != 0 && (c >> 8) == grid) return (int)(c & 0xff);
  int cl = 1;
  if (grid % 4 == 0 && cluster_fits<4>(grid)) cl = 4;
  else if (grid % 2 == 0 && cluster_fits<2>(grid)) cl = 2;
  cache[dev].store(((long long)grid << 8) | cl);
  return cl;
}

template <int LP, int CL>
static cudaError_t lag_project_cl(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                                  const double* U, const double* Z, double* partS, double* partT, int* state) {
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = smem_attr_once(attr, (const void*)gs_lag_project_kernel<LP, CL>, (int)gs_lag_smem());
  if (e != cudaSuccess) return e;
  if (CL == 1)
    return launch_pdl(gs_lag_project_kernel<LP, CL>, dim3(p.grid), dim3(kLagThreads), gs_lag_smem(), st, V, L, ncols,
                      n, U, Z, partS, partT, state);
  return launch_pdl_cluster(gs_lag_project_kernel<LP, CL>, dim3(p.grid), dim3(kLagThreads), CL, gs_lag_smem(), st, V,
                            L, ncols, n, U, Z, partS, partT, state);
}

template <int LP>
static cudaError_t lag_project_lp(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                                  const double* U, const double* Z, double* partS, double* partT, int* state) {
  const int cl = lag_cluster(p.grid);
  if (cl == 4) return lag_project_cl<LP, 4>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
  if (cl == 2) return lag_project_cl<LP, 2>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
  return lag_project_cl<LP, 1>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
}

int gs_lag_rows(const GsPlan& p) { return p.grid / lag_cluster(p.grid); }

template <int LP>
static cudaError_t lag_correct_lp(const GsPlan& p, cudaStream_t st, double* V, VLayout L, int ncols, int n, double* R,
                                  const double* Z, const double* partS, const double* partT, int nrows_in,
                                  double* part_out, double* scal, double* alpha, double* beta, int* state) {
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = smem_attr_once(attr, (const void*)gs_lag_correct_kernel<LP>, (int)gs_lag_smem());
  if (e != cudaSuccess) return e;
  return launch_pdl(gs_lag_correct_kernel<LP>, dim3(p.grid), dim3(kLagThreads), gs_lag_smem(), st, V, L, ncols, n, R,
                    Z, partS, partT, nrows_in, part_out, scal, alpha, beta, state);
}

cudaError_t gs_lag_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                           const double* U, const double* Z, double* partS, double* partT, int* state) {
  if (ncols <= 32) return lag_project_lp<4>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
  if (ncols <= 64) return lag_project_lp<8>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
  return lag_project_lp<16>(p, st, V, L, ncols, n, U, Z, partS, partT, state);
}

cudaError_t gs_lag_correct(const GsPlan& p, cudaStream_t st, double* V, VLayout L, int ncols, int n, double* R,
                           const double* Z, const double* partS, const double* partT, int nrows_in,
                           double* part_out, double* scal, double* alpha, double* beta, int* state) {
  if (ncols <= 32)
    return lag_correct_lp<4>(p, st, V, L, ncols, n, R, Z, partS, partT, nrows_in, part_out, scal, alpha, beta, state);
  if (ncols <= 64)
    return lag_correct_lp<8>(p, st, V, L, ncols, n, R, Z, partS, partT, nrows_in, part_out, scal, alpha, beta, state);
  return lag_correct_lp<16>(p, st, V, L, ncols, n, R, Z, partS, partT, nrows_in, part_out, scal, alpha, beta, state);
}

}  // namespace lg
