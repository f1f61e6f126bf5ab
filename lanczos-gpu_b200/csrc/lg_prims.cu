// lg_prims.cu — stand-alone C ABI primitives built on the eigsh kernels.
//
// lg_cgs2_orthogonalize: two classical Gram-Schmidt passes of a vector
// against the first ncols columns of a row-major basis — the reference's
// cgs_orthogonalize + dgks_reorth (src/lanczos_ops.cuh:113-192) as one call on
// device pointers and the caller's stream, running the three fused passes of
// the Lanczos step (lg_gs.cu) plus a one-CTA finalisation.
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_solver.h"

#include <string>

namespace lg {

// coef = h1 + s; norms = (||w||, ||r1||, ||r2||) from the three partial blocks.
__global__ void __launch_bounds__(kGsThreads, 1)
cgs2_finalize_kernel(const double* __restrict__ partA, const double* __restrict__ partB,
                     const double* __restrict__ partC, int nrows, int ncols, double* coef, double* norms,
                     const int* state) {
  __shared__ double red[kGsThreads];
  __shared__ double h1[kMaxCols], s[kMaxCols];
  __shared__ double scr[32];
  double wn2, r1n2, dummy;
  reduce_partials(partA, nrows, ncols, h1, &wn2, red);
  reduce_partials(partB, nrows, ncols, s, &r1n2, red);
  double r2 = 0.0;
  for (int i = threadIdx.x; i < nrows; i += blockDim.x) r2 += partC[(size_t)i * kPartStride + kPartScalar];
  r2 = block_sum(r2, scr);
  (void)dummy;
  if (threadIdx.x < ncols) coef[threadIdx.x] = h1[threadIdx.x] + s[threadIdx.x];
  if (threadIdx.x == 0) {
    const bool ok = state[ST_STATUS] == STATUS_RUNNING;
    norms[0] = ok ? sqrt(wn2) : NAN;
    norms[1] = ok ? sqrt(r1n2) : NAN;
    norms[2] = ok ? sqrt(r2) : NAN;
  }
}

// Number of doubles of workspace for `grid` CTAs: three partial blocks and the
// scalar words; the int state words follow (ST_WORDS ints).
size_t cgs2_workspace_doubles(int grid) { return (size_t)3 * grid * kPartStride + SC_WORDS; }

int cgs2_run(const double* V, int ldv, int n, int ncols, const double* w, double* r, double* coef, double* norms,
             cudaStream_t st, int grid, double* ws, int* state) {
  const GsPlan p = gs_plan(n, ncols, grid);
  VLayout L;   // the caller's row-major basis
  L.rs = ldv;
  L.ps = 8;
  double* partA = ws;
  double* partB = ws + (size_t)grid * kPartStride;
  double* partC = ws + (size_t)2 * grid * kPartStride;
  double* scal = ws + (size_t)3 * grid * kPartStride;
  cudaError_t e = cudaMemsetAsync(state, 0, sizeof(int) * ST_WORDS, st);
  if (e == cudaSuccess) e = gs_project(p, st, V, L, ncols, n, w, partA, state);
  if (e == cudaSuccess) e = gs_correct_project(p, st, V, L, ncols, n, w, r, partA, p.grid, partB, scal, state);
  if (e == cudaSuccess)
    e = gs_correct(p, st, V, L, ncols, n, r, partB, p.grid, partC, scal, nullptr, 0, 0, state);
  if (e == cudaSuccess) {
    cgs2_finalize_kernel<<<1, kGsThreads, 0, st>>>(partA, partB, partC, p.grid, ncols, coef, norms, state);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    g_last_error = std::string("CUDA error ") + cudaGetErrorString(e) + " in lg_cgs2_orthogonalize";
    return LG_ERR_CUDA;
  }
  return LG_OK;
}

int cgs2_check_args(const double* V, int ldv, int n, int ncols, const double* w, double* r, double* coef,
                    double* norms) {
  if (!V || !w || !r || !coef || !norms || n < 1 || ncols < 1 || ncols > kMaxCols || ldv < ncols + (ncols & 1)) {
    g_last_error = "lg_cgs2_orthogonalize: need device pointers, n >= 1, 1 <= ncols <= 128, ldv >= ncols rounded "
                   "up to even";
    return LG_ERR_INVALID;
  }
  if (w == r) {
    g_last_error = "lg_cgs2_orthogonalize: r must not alias w";
    return LG_ERR_INVALID;
  }
  if (((uintptr_t)V & 15u) != 0 || (ldv & 1)) {
    g_last_error = "lg_cgs2_orthogonalize: V must be 16-byte aligned with an even ldv";
    return LG_ERR_INVALID;
  }
  return LG_OK;
}

int cgs2_grid() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

}  // namespace lg

extern "C" int lg_cgs2_orthogonalize(const double* V, int ldv, int n, int ncols, const double* w, double* r,
                                     double* coef, double* norms, void* stream) {
  using namespace lg;
  int rc = cgs2_check_args(V, ldv, n, ncols, w, r, coef, norms);
  if (rc != LG_OK) return rc;
  const int grid = cgs2_grid();
  if (grid < 1) {
    g_last_error = "lg_cgs2_orthogonalize: no CUDA device";
    return LG_ERR_CUDA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t nd = cgs2_workspace_doubles(grid);
  void* ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, sizeof(double) * nd + sizeof(int) * ST_WORDS, st);
  if (e != cudaSuccess) {
    g_last_error = std::string("lg_cgs2_orthogonalize: ") + cudaGetErrorString(e);
    return LG_ERR_NOMEM;
  }
  double* wsd = static_cast<double*>(ws);
  rc = cgs2_run(V, ldv, n, ncols, w, r, coef, norms, st, grid, wsd, reinterpret_cast<int*>(wsd + nd));
  cudaFreeAsync(ws, st);
  return rc;
}
