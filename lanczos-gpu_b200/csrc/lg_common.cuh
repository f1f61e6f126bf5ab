// lg_common.cuh — shared constants, error handling and sm_100a device helpers
// for the B200 Lanczos engine.
//
// Numerical constants restate the reference's choices
// (src/lanczos_types.cuh:63-75): DGKS threshold 1/sqrt(2), SAFE_MIN = DBL_MIN,
// MACH_EPS = DBL_EPSILON, at most two refinement passes.
#pragma once

#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cfloat>

namespace lg {

// ---------------------------------------------------------------------------
// Limits and layout constants
// ---------------------------------------------------------------------------
constexpr int kMaxCols = 128;          // basis columns held in one tile (ncv+1 <= 128)
constexpr int kPartStride = 136;       // doubles per partial-sum row: 128 columns + scalars
constexpr int kPartScalar = 128;       // slot of the first scalar in a partial row
constexpr int kRowAlign = 256;         // leading dimension of V is a multiple of this
constexpr int kGsThreads = 1024;       // threads of the Gram-Schmidt pass kernels (one CTA per SM)

constexpr double kDgks = 0.7071067811865476;      // 1/sqrt(2)
constexpr double kSafeMin = DBL_MIN;
constexpr double kEps = DBL_EPSILON;

// Device-side state words (int32 array in device memory).
enum StateWord {
  ST_STATUS = 0,      // 0 = running; otherwise one of Status
  ST_STEP = 1,        // step index the status refers to
  ST_NCONV = 2,
  ST_NEV_USE = 3,
  ST_DONE = 4,        // restart kernel decided to stop (converged or out of iterations)
  ST_KSEL = 5,        // number of selected Ritz pairs written to zsel
  ST_ERRINFO = 6,     // extra error detail (e.g. tridiagonal QR failure, timeout site)
  ST_WORDS = 16
};

enum Status {
  STATUS_RUNNING = 0,
  STATUS_PASS3 = 1,       // DGKS wants a third Gram-Schmidt pass at step ST_STEP
  STATUS_BREAKDOWN = 2,   // invariant subspace found after step ST_STEP
  STATUS_TRIDIAG_FAIL = 3,
  STATUS_TIMEOUT = 4,     // a bounded device-side wait gave up
  STATUS_PASS3_LAG = 5,   // a delayed second pass (lag step) left too little of the residual of step ST_STEP:
                          // apply that pass explicitly, then a third, as DGKS does
};

// Device-side double scalars.
enum ScalarWord {
  SC_WN2 = 0,        // ||w||^2 of the current step
  SC_R1N2 = 1,       // ||r1||^2 after the first Gram-Schmidt pass
  SC_HJ = 2,         // first-pass coefficient h_j (diagonal part of alpha_j)
  SC_RCOEF = 3,      // restart: coefficient on the old residual
  SC_TAU = 4,        // restart: coefficient on V_new[:, nev_use]
  SC_BN = 5,         // residual norm at the last restart check
  SC_BETA_NEXT = 6,  // norm of the residual that will become the next basis vector
  SC_ALPHA_PREV = 7, // lag step j: alpha_{j-1} before its delayed second-pass term (read by every CTA)
  SC_WORDS = 16
};

__host__ __device__ inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------------------
// Warp / block reductions (fixed order, so every run is bitwise repeatable)
// ---------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_sumf(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum one double over the block; result valid in every thread.
// `scratch` needs blockDim.x/32 doubles.
__device__ inline double block_sum(double v, double* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < nw; ++w) t += scratch[w];
  __syncthreads();
  return t;
}

// Reference: src/lanczos_ops.cuh:264-277 (adaptive_breakdown_tol), evaluated
// for the step that produced the residual (index jr): eps^(2/3) times the
// largest absolute row sum of the tridiagonal T[0..jr], with alpha[jr] taken
// as `alpha_last` when `use_last` (a lag step checks with the corrected value
// before it is stored).  Called by all 32 lanes of a warp (one row per lane,
// max-reduced by shuffles: the same value as a serial scan); the result is
// valid in every lane.
__device__ inline double breakdown_tol_warp(const double* alpha, const double* beta, int jr, bool use_last = false,
                                            double alpha_last = 0.0) {
  double est = 0.0;
  for (int i = threadIdx.x & 31; i <= jr; i += 32) {
    double rs = fabs((use_last && i == jr) ? alpha_last : alpha[i]);
    if (i > 0) rs += fabs(beta[i]);
    if (i < jr) rs += fabs(beta[i + 1]);
    est = fmax(est, rs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) est = fmax(est, __shfl_xor_sync(0xffffffffu, est, o));
  const double eps23 = 3.6687695461231177e-11;  // DBL_EPSILON^(2/3)
  return eps23 * fmax(est, kSafeMin);
}

// ---------------------------------------------------------------------------
// Partial-sum rows (one per CTA, kPartStride doubles: columns then scalars)
// ---------------------------------------------------------------------------
// Reduce `nrows` partial rows: columns [0, nc) into out[0..nc), the scalar
// slot into *scal_out.  Every thread of the block gets the same values.
// `red` needs blockDim.x doubles; blockDim.x must be a multiple of 128.
// Rows are summed in order r = grp, grp + ngrp, ... by every thread; the loads
// go out eight at a time (independent), the adds keep that order, so the
// result does not depend on the batching.
__device__ __forceinline__ double sum_rows_strided(const double* __restrict__ part, int nrows, int first, int stride,
                                                   int slot) {
  double acc = 0.0;
  int r = first;
  for (; r + 7 * stride < nrows; r += 8 * stride) {
    double v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = part[(size_t)(r + u * stride) * kPartStride + slot];
#pragma unroll
    for (int u = 0; u < 8; ++u) acc += v[u];
  }
  for (; r < nrows; r += stride) acc += part[(size_t)r * kPartStride + slot];
  return acc;
}

__device__ inline void reduce_partials(const double* __restrict__ part, int nrows, int nc, double* out,
                                double* scal_out, double* red) {
  const int t = threadIdx.x;
  const int ngrp = blockDim.x >> 7;
  const int slot = t & 127, grp = t >> 7;
  double acc = 0.0;
  if (slot < nc) acc = sum_rows_strided(part, nrows, grp, ngrp, slot);
  red[grp * 128 + slot] = acc;
  double sc = 0.0;
  if (t < 32) {
    sc = sum_rows_strided(part, nrows, t, 32, kPartScalar);
    sc = warp_sum(sc);
  }
  __syncthreads();
  if (t < nc) {
    double s = 0.0;
    for (int g = 0; g < ngrp; ++g) s += red[g * 128 + t];
    out[t] = s;
  }
  if (t == 0) *scal_out = sc;
  __syncthreads();
}

// reduce_partials of two tables with the same row count in one pass (their
// loads in flight together); same values as two separate calls.  `red`
// needs 2 * blockDim.x doubles.
__device__ inline void reduce_partials2(const double* __restrict__ pa, const double* __restrict__ pb, int nrows,
                                        int nca, int ncb, double* outa, double* outb, double* sca_out,
                                        double* scb_out, double* red) {
  const int t = threadIdx.x;
  const int ngrp = blockDim.x >> 7;
  const int slot = t & 127, grp = t >> 7;
  double acca = 0.0, accb = 0.0;
  if (slot < nca) acca = sum_rows_strided(pa, nrows, grp, ngrp, slot);
  if (slot < ncb) accb = sum_rows_strided(pb, nrows, grp, ngrp, slot);
  red[grp * 128 + slot] = acca;
  red[blockDim.x + grp * 128 + slot] = accb;
  double sca = 0.0, scb = 0.0;
  if (t < 32) {
    sca = warp_sum(sum_rows_strided(pa, nrows, t, 32, kPartScalar));
    scb = warp_sum(sum_rows_strided(pb, nrows, t, 32, kPartScalar));
  }
  __syncthreads();
  if (t < nca) {
    double s = 0.0;
    for (int g = 0; g < ngrp; ++g) s += red[g * 128 + t];
    outa[t] = s;
  }
  if (t < ncb) {
    double s = 0.0;
    for (int g = 0; g < ngrp; ++g) s += red[blockDim.x + g * 128 + t];
    outb[t] = s;
  }
  if (t == 0) {
    *sca_out = sca;
    *scb_out = scb;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Safe scaling (two-step when the norm is below SAFE_MIN; the reference does
// the same with two Dscal calls, src/lanczos_ops.cuh:204-216).
// x * s1 * s2 where s2 == 1 in the normal case.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void safe_inv(double nrm, double& s1, double& s2) {
  if (nrm >= kSafeMin) { s1 = 1.0 / nrm; s2 = 1.0; }
  else if (nrm > 0.0) { s1 = kSafeMin / nrm; s2 = 1.0 / kSafeMin; }
  else { s1 = 1.0; s2 = 1.0; }
}

// ---------------------------------------------------------------------------
// Counter-based uniform RNG (splitmix64 finaliser).  Used for the default
// starting vector and for restart vectors after an invariant subspace.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// uniform in [-0.5, 0.5)
__host__ __device__ __forceinline__ double uniform_centered(uint64_t seed, uint64_t i) {
  uint64_t r = mix64(seed * 0x100000001B3ull + mix64(i));
  return (double)(r >> 11) * (1.0 / 9007199254740992.0) - 0.5;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (the Lanczos step kernels).  A kernel launched
// with launch_pdl may start while the kernel before it on the stream is still
// finishing; griddep_wait() blocks until that kernel has completed and its
// memory is visible, so everything the previous kernel writes is read after
// it.  griddep_launch_dependents() lets the next kernel of the stream start
// early (its own griddep_wait still waits for this one to complete).  Both
// are no-ops in a kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_pdl for a kernel launched in clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, int cluster, size_t smem,
                                      cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// Dynamic shared memory above the 48 KB default must be opted into per kernel
// and per device.  `done` is the caller's bit set of devices (ids 0..63) on
// which the attribute is already set; devices beyond 63 set it on every call.
// Two threads racing on a first call both set it, which is harmless.
// ---------------------------------------------------------------------------
inline cudaError_t smem_attr_once(std::atomic<unsigned long long>& done, const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Resident CTAs of `threads` threads per SM for `kernel` on the current
// device (no dynamic shared memory), queried once per device and cached in
// `cache` (one entry per device ordinal; 0 = not yet known).  Falls back to
// `fallback` when the query fails.
struct OccupancyCache {
  std::atomic<int> blocks[64] = {};
};
inline int resident_blocks_once(OccupancyCache& cache, const void* kernel, int threads, int fallback) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fallback;
  int b = cache.blocks[dev].load(std::memory_order_acquire);
  if (b > 0) return b;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0) != cudaSuccess || b < 1) {
    (void)cudaGetLastError();
    return fallback;
  }
  cache.blocks[dev].store(b, std::memory_order_release);
  return b;
}

}  // namespace lg
