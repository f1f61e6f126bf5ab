// lg_spmv.cu — CSR SpMV for the Lanczos step, plus small vector kernels.
//
// Replaces the operator layer of the reference (src/matvec_operator.cuh:56-135:
// cuSPARSE SpMV, and the mixed fp32 path with its two cast kernels
// src/cast_kernels.cu:7-15).  Here:
//   * one kernel per step does  beta_j = ||r||, v_j = r / beta_j,
//     w = A v_j  — the normalisation of the previous residual is folded into
//     the SpMV (w = (A r) / beta_j), so no separate scale/copy launches; in a
//     lag step (BETA_LAG, Vj null) only w = A r / ||r|| (v_j is finished by
//     the delayed second Gram-Schmidt pass, lg_gs.cu);
//   * the fp32-value variant keeps x and the accumulator in fp64
//     (fp32 values halve the value stream; accuracy stays fp64);
//   * rows are handled by a group of L lanes (vector-per-row, L picked from
//     the mean row length), lanes read consecutive nonzeros (coalesced).
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_csr.cuh"

#include <cmath>

namespace lg {

// Prologue shared by the SpMV step and the normalise-only step: reduce the
// norm partials of R, run the DGKS / breakdown checks, store beta_j.  Every
// CTA computes the same values in the same order; block 0 publishes them.
// Returns the block-uniform stop code; s1*s2 is the safe 1/||R||.
__device__ int step_prologue(const double* __restrict__ part_in, int nrows_in, int j, int beta_mode,
                             double* alpha, double* beta, double* scal, int* state, double& s1o, double& s2o) {
  __shared__ double sh_s1, sh_s2;
  __shared__ int sh_stop;
  if (threadIdx.x < 32) {
    double nrm2 = 0.0;
#pragma unroll 4
    for (int r = threadIdx.x; r < nrows_in; r += 32) nrm2 += part_in[(size_t)r * kPartStride + kPartScalar];
    nrm2 = warp_sum(nrm2);
    const double btol =
        (beta_mode == BETA_STEP || beta_mode == BETA_RESTART) ? breakdown_tol_warp(alpha, beta, j - 1) : 0.0;
    if (threadIdx.x == 0) {
      const double bn = sqrt(nrm2);
      int stop = STATUS_RUNNING;
      if (beta_mode == BETA_STEP) {
        if (nrm2 <= 0.5 * scal[SC_R1N2]) stop = STATUS_PASS3;
        else if (bn < btol) stop = STATUS_BREAKDOWN;
      } else if (beta_mode == BETA_RESTART) {
        if (bn < btol) stop = STATUS_BREAKDOWN;
      }
      double s1, s2;
      safe_inv(bn, s1, s2);
      sh_s1 = s1;
      sh_s2 = s2;
      sh_stop = stop;
      if (blockIdx.x == 0) {
        if (stop != STATUS_RUNNING) {
          state[ST_STEP] = j - 1;
          state[ST_STATUS] = stop;
        } else {
          if (beta_mode == BETA_STEP || beta_mode == BETA_RESTART) beta[j] = bn;
          else if (beta_mode == BETA_ZERO) beta[j] = 0.0;
          else if (beta_mode == BETA_LAG) scal[SC_ALPHA_PREV] = alpha[j - 1];
          scal[SC_BETA_NEXT] = bn;
        }
      }
    }
  }
  __syncthreads();
  s1o = sh_s1;
  s2o = sh_s2;
  return sh_stop;
}

// `list` (optional, `count` entries): the rows to process, else rows 0..count-1.
template <typename VT, int L>
__global__ void __launch_bounds__(256)
spmv_step_kernel(int count, const int* __restrict__ list, const int* __restrict__ rowptr,
                 const int* __restrict__ col, const VT* __restrict__ val, const double* __restrict__ R,
                 const double* __restrict__ R_own, double* __restrict__ W, double* __restrict__ Vj, int ldv,
                 const double* __restrict__ part_in, int nrows_in, int j, int beta_mode, double* alpha,
                 double* beta, double* scal, int* state) {
  griddep_wait();   // R and the partial sums come from the previous kernel
  griddep_launch_dependents();
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  double s1, s2;
  if (step_prologue(part_in, nrows_in, j, beta_mode, alpha, beta, scal, state, s1, s2) != STATUS_RUNNING) return;

  // Each lane group works on two rows at once so the dependent load chains
  // (row_ptr -> col -> x gather) of the two rows overlap; the row bounds of
  // the next trip are loaded while this trip's gathers are in flight.
  const int lane = threadIdx.x & (L - 1);
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  const int rows_per_warp = 32 / L;
  const int gl = (threadIdx.x & 31) / L;
  auto bounds = [&](int w, int& rowA, int& rowB, int& kA, int& eA, int& kB, int& eB) {
    const int iA = w * rows_per_warp * 2 + gl, iB = iA + rows_per_warp;
    const bool okA = iA < count, okB = iB < count;
    rowA = okA ? (list ? __ldg(list + iA) : iA) : -1;
    rowB = okB ? (list ? __ldg(list + iB) : iB) : -1;
    kA = eA = kB = eB = 0;
    if (okA) { kA = __ldg(rowptr + rowA); eA = min(__ldg(rowptr + rowA + 1), kA + kLongRow); kA += lane; }
    if (okB) { kB = __ldg(rowptr + rowB); eB = min(__ldg(rowptr + rowB + 1), kB + kLongRow); kB += lane; }
  };
  int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int rowA, rowB, kA, eA, kB, eB;
  if ((long long)w * rows_per_warp * 2 < count) bounds(w, rowA, rowB, kA, eA, kB, eB);
  // U nonzeros per lane and row are loaded before any of their gathers is
  // issued (U * L per row per trip), so rows of hundreds of nonzeros keep
  // 2U gathers per lane in flight; each lane still adds its nonzeros
  // k, k + L, k + 2L, ... in that order.
  constexpr int U = L >= 32 ? 4 : (L >= 16 ? 2 : 1);
  for (; (long long)w * rows_per_warp * 2 < count; w += warps_total) {
    double accA = 0.0, accB = 0.0;
    while (kA < eA || kB < eB) {
      int cA[U], cB[U];
      VT vA[U], vB[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int ka = kA + u * L, kb = kB + u * L;
        cA[u] = ka < eA ? __ldg(col + ka) : -1;
        vA[u] = ka < eA ? __ldg(val + ka) : VT(0);
        cB[u] = kb < eB ? __ldg(col + kb) : -1;
        vB[u] = kb < eB ? __ldg(val + kb) : VT(0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (cA[u] >= 0) accA += (double)vA[u] * __ldg(R + cA[u]);
        if (cB[u] >= 0) accB += (double)vB[u] * __ldg(R + cB[u]);
      }
      kA += U * L;
      kB += U * L;
    }
    const int curA = rowA, curB = rowB;
    const int wn = w + warps_total;
    if ((long long)wn * rows_per_warp * 2 < count) bounds(wn, rowA, rowB, kA, eA, kB, eB);
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) {
      accA += __shfl_xor_sync(0xffffffffu, accA, o);
      accB += __shfl_xor_sync(0xffffffffu, accB, o);
    }
    if (lane == 0) {
      if (curA >= 0) {
        W[curA] = (accA * s1) * s2;
        if (Vj) Vj[(size_t)curA * ldv] = (R_own[curA] * s1) * s2;
      }
      if (curB >= 0) {
        W[curB] = (accB * s1) * s2;
        if (Vj) Vj[(size_t)curB * ldv] = (R_own[curB] * s1) * s2;
      }
    }
  }
}

__global__ void __launch_bounds__(256)
normalize_step_kernel(int n, const double* __restrict__ R, double* __restrict__ Vj, int ldv, double* __restrict__ out,
                      const double* __restrict__ part_in, int nrows_in, int j, int beta_mode, double* alpha,
                      double* beta, double* scal, int* state) {
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  double s1, s2;
  if (step_prologue(part_in, nrows_in, j, beta_mode, alpha, beta, scal, state, s1, s2) != STATUS_RUNNING) return;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
  {
    const double v = (R[i] * s1) * s2;
    Vj[(size_t)i * ldv] = v;
    if (out) out[i] = v;
  }
}

cudaError_t normalize_step(cudaStream_t st, int grid, int n, const double* R, double* Vj, int ldv, double* out,
                           const double* part_in,
                           int nrows_in, int j, int beta_mode, double* alpha, double* beta, double* scal,
                           int* state) {
  normalize_step_kernel<<<grid, 256, 0, st>>>(n, R, Vj, ldv, out, part_in, nrows_in, j, beta_mode, alpha, beta, scal,
                                              state);
  return cudaGetLastError();
}

template <typename VT, int L>
__global__ void __launch_bounds__(256)
spmv_plain_kernel(int n, const int* __restrict__ rowptr, const int* __restrict__ col,
                  const VT* __restrict__ val, const double* __restrict__ x, double* __restrict__ y,
                  double shift) {
  const int lane = threadIdx.x & (L - 1);
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  const int rows_per_warp = 32 / L;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; (long long)w * rows_per_warp < n;
       w += warps_total) {
    const int row = w * rows_per_warp + ((threadIdx.x & 31) / L);
    const bool valid = row < n;
    const double acc = row_dot<VT, L>(rowptr, col, val, x, row, valid, lane, true);
    if (valid && lane == 0) y[row] = acc + shift * x[row];
  }
}

// Remainders of the long rows: one warp per chunk of kLongRow nonzeros.
template <typename VT>
__global__ void __launch_bounds__(256)
long_chunk_kernel(int nchunks, const int* __restrict__ cb, const int* __restrict__ ce, const int* __restrict__ col,
                  const VT* __restrict__ val, const double* __restrict__ x, double* __restrict__ csum,
                  const int* __restrict__ state) {
  if (state && state[ST_STATUS] != STATUS_RUNNING) return;
  const int lane = threadIdx.x & 31;
  for (int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks; c += (gridDim.x * blockDim.x) >> 5) {
    // four nonzeros per lane are loaded before their gathers are issued; the
    // lane adds them in index order
    double acc = 0.0;
    const int e = ce[c];
    for (int k = cb[c] + lane; k < e; k += 128) {
      int cc[4];
      VT vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        cc[u] = k + 32 * u < e ? __ldg(col + k + 32 * u) : -1;
        vv[u] = k + 32 * u < e ? __ldg(val + k + 32 * u) : VT(0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (cc[u] >= 0) acc += (double)vv[u] * __ldg(x + cc[u]);
    }
    acc = warp_sum(acc);
    if (lane == 0) csum[c] = acc;
  }
}

// y[row] += (sum of its chunks, in chunk order) / ||r|| for the Lanczos step
// (scal: the norm published by the step's prologue), or unscaled.
__global__ void long_combine_kernel(int nlong, const int* __restrict__ rows, const int* __restrict__ first,
                                    const double* __restrict__ csum, double* __restrict__ y,
                                    const double* __restrict__ scal, const int* __restrict__ state) {
  if (state && state[ST_STATUS] != STATUS_RUNNING) return;
  double s1 = 1.0, s2 = 1.0;
  if (scal) safe_inv(scal[SC_BETA_NEXT], s1, s2);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nlong; i += gridDim.x * blockDim.x) {
    double acc = 0.0;
    for (int c = first[i]; c < first[i + 1]; ++c) acc += csum[c];
    y[rows[i]] += (acc * s1) * s2;
  }
}

template <typename VT>
static cudaError_t long_rows_finish(const CsrDev& A, const VT* val, cudaStream_t st, const double* x, double* y,
                                    const double* scal, const int* state) {
  if (A.nlong == 0) return cudaSuccess;
  int grid = (A.nchunks * 32 + 255) / 256;
  if (grid > 4096) grid = 4096;
  long_chunk_kernel<VT><<<grid, 256, 0, st>>>(A.nchunks, A.chunk_begin, A.chunk_end, A.col, val, x, A.chunk_sum,
                                              state);
  long_combine_kernel<<<(A.nlong + 255) / 256, 256, 0, st>>>(A.nlong, A.long_rows, A.long_first, A.chunk_sum, y,
                                                             scal, state);
  return cudaGetLastError();
}

template <typename VT>
static cudaError_t launch_step(const CsrDev& A, const VT* val, cudaStream_t st, int grid, const double* R,
                               const double* R_own, double* W, double* Vj, int ldv, const double* part_in,
                               int nrows_in, int j, int beta_mode, double* alpha, double* beta, double* scal,
                               int* state) {
  // `grid` is 8 CTAs per SM; kernels whose registers allow fewer resident
  // CTAs get one full wave of them instead (the loop over rows is
  // grid-strided, so CTAs that could not start at once would only add a tail)
#define LG_STEP(LN, CNT, LIST)                                                                              \
  do {                                                                                                      \
    static OccupancyCache occ_;                                                                             \
    const int res_ = resident_blocks_once(occ_, (const void*)spmv_step_kernel<VT, LN>, 256, 8);             \
    const int g_ = res_ < 8 ? grid / 8 * res_ : grid;                                                       \
    cudaError_t e_ = launch_pdl(spmv_step_kernel<VT, LN>, dim3(g_), dim3(256), 0, st, CNT, LIST, A.rowptr,    \
                                A.col, val, R, R_own, W, Vj, ldv, part_in, nrows_in, j, beta_mode, alpha, beta, \
                                scal, state);                                                                \
    if (e_ != cudaSuccess) return e_;                                                                       \
  } while (0)
  const int ncls = A.nclasses > 0 ? A.nclasses : 1;
  for (int c = 0; c < ncls; ++c) {
    const int lanes = A.nclasses > 0 ? A.class_lanes[c] : A.lanes;
    const int cnt = A.nclasses > 0 ? A.class_count[c] : A.n;
    const int* list = A.nclasses > 0 ? A.class_rows[c] : nullptr;
    switch (lanes) {
      case 2: LG_STEP(2, cnt, list); break;
      case 4: LG_STEP(4, cnt, list); break;
      case 8: LG_STEP(8, cnt, list); break;
      case 16: LG_STEP(16, cnt, list); break;
      default: LG_STEP(32, cnt, list); break;
    }
  }
#undef LG_STEP
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return long_rows_finish<VT>(A, val, st, R, W, scal, state);
}

cudaError_t spmv_step(const CsrDev& A, cudaStream_t st, int grid, const double* R, double* W, double* Vj,
                      int ldv, const double* part_in, int nrows_in, int j, int beta_mode, double* alpha,
                      double* beta, double* scal, int* state, const double* R_own) {
  if (!R_own) R_own = R;
  if (A.val32)
    return launch_step<float>(A, A.val32, st, grid, R, R_own, W, Vj, ldv, part_in, nrows_in, j, beta_mode, alpha,
                              beta, scal, state);
  return launch_step<double>(A, A.val64, st, grid, R, R_own, W, Vj, ldv, part_in, nrows_in, j, beta_mode, alpha,
                             beta, scal, state);
}

template <typename VT>
static cudaError_t launch_plain(const CsrDev& A, const VT* val, cudaStream_t st, int grid, const double* x,
                                double* y, double shift) {
#define LG_PLAIN(LN) \
  spmv_plain_kernel<VT, LN><<<grid, 256, 0, st>>>(A.n, A.rowptr, A.col, val, x, y, shift)
  switch (A.lanes) {
    case 2: LG_PLAIN(2); break;
    case 4: LG_PLAIN(4); break;
    case 8: LG_PLAIN(8); break;
    case 16: LG_PLAIN(16); break;
    default: LG_PLAIN(32); break;
  }
#undef LG_PLAIN
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return long_rows_finish<VT>(A, val, st, x, y, nullptr, nullptr);
}

cudaError_t spmv_plain(const CsrDev& A, cudaStream_t st, int grid, const double* x, double* y,
                       double shift) {
  if (A.val32) return launch_plain<float>(A, A.val32, st, grid, x, y, shift);
  return launch_plain<double>(A, A.val64, st, grid, x, y, shift);
}

// ---------------------------------------------------------------------------
// x[i] = uniform(seed, index0 + i): a row-partitioned vector is the slice of
// the same global vector on every partition.
__global__ void fill_random_kernel(double* x, int n, int ld, uint64_t seed, long long index0) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ld; i += gridDim.x * blockDim.x)
    x[i] = (i < n) ? uniform_centered(seed, (uint64_t)(index0 + i)) : 0.0;
}

cudaError_t fill_random(cudaStream_t st, double* x, int n, int ld, uint64_t seed, long long index0) {
  int grid = (ld + 255) / 256;
  if (grid > 4096) grid = 4096;
  fill_random_kernel<<<grid, 256, 0, st>>>(x, n, ld, seed, index0);
  return cudaGetLastError();
}

__global__ void norm_partials_kernel(const double* __restrict__ x, int ld, double* __restrict__ part_out) {
  __shared__ double scr[32];
  const long long b = (long long)ld * blockIdx.x / gridDim.x;
  const long long e = (long long)ld * (blockIdx.x + 1) / gridDim.x;
  double acc = 0.0;
  for (long long i = b + threadIdx.x; i < e; i += blockDim.x) acc += x[i] * x[i];
  acc = block_sum(acc, scr);
  if (threadIdx.x == 0) part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = acc;
}

cudaError_t norm_partials(cudaStream_t st, int grid, const double* x, int ld, double* part_out) {
  norm_partials_kernel<<<grid, 256, 0, st>>>(x, ld, part_out);
  return cudaGetLastError();
}

}  // namespace lg
