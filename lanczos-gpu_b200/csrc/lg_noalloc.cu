// lg_noalloc.cu — lg_cgs2_orthogonalize_noalloc: the CGS2 primitive for
// callers that must not allocate device memory.
//
// Who needs it: code that cannot call cudaMalloc/cudaFree at the point where
// it re-orthogonalises a vector — for example a routine invoked from inside a
// custom device-memory allocator or memory-pool hook (calling back into the
// allocator there would recurse), or a service that reserves its whole device
// memory budget at start-up and must not grow or fragment it afterwards.
// lg_cgs2_orthogonalize takes a stream-ordered allocation for its partial
// sums on every call; this variant takes none.
//
// How: its workspace is the file-scope array g_cgs2_scratch below, a fixed
// 0.5 MiB of device memory that every GPU which loads this library keeps until
// the process exits.  Device code could name the array directly, but the host
// must not pass its name to a kernel (in host code it is only a stand-in, not
// a device address): the first call on each device resolves the real address
// with cudaGetSymbolAddress while that device is current, checks the result
// and caches it.  Under CUDA's lazy module loading that first call is also
// when this library's device code is loaded on the device (driver memory is
// taken then), so it belongs outside the no-allocation context, and before
// any stream capture.  A cudaDeviceReset invalidates the cached address.
//
// Every call on a device shares the one array, and the array keeps whatever
// the previous call left in it: the status words are cleared at the start of
// each call, everything else is written before it is read.  Two calls whose
// work overlaps on the GPU (different streams, or host threads sharing a
// device without ordering their streams) race on the array and corrupt each
// other's results — order them on one stream.
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_solver.h"

#include <mutex>
#include <string>

namespace lg {

int cgs2_run(const double* V, int ldv, int n, int ncols, const double* w, double* r, double* coef, double* norms,
             cudaStream_t st, int grid, double* ws, int* state);
int cgs2_check_args(const double* V, int ldv, int n, int ncols, const double* w, double* r, double* coef,
                    double* norms);
size_t cgs2_workspace_doubles(int grid);
int cgs2_grid();

namespace {

constexpr int kNoAllocMaxGrid = 160;   // CTAs the fixed workspace is sized for (B200 has 148 SMs)
constexpr size_t kNoAllocDoubles = (size_t)3 * kNoAllocMaxGrid * kPartStride + SC_WORDS + ST_WORDS;

static __device__ __align__(256) double g_cgs2_scratch[kNoAllocDoubles];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
double* g_scratch_addr[kMaxDevices] = {};

// Device address of g_cgs2_scratch on the current device (resolved once).
int scratch_address(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    g_last_error = "lg_cgs2_orthogonalize_noalloc: no usable current CUDA device";
    return LG_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_cgs2_scratch);
    if (e != cudaSuccess || p == nullptr) {
      g_last_error = std::string("lg_cgs2_orthogonalize_noalloc: cudaGetSymbolAddress failed: ") +
                     cudaGetErrorString(e);
      return LG_ERR_CUDA;
    }
    g_scratch_addr[dev] = static_cast<double*>(p);
  }
  *out = g_scratch_addr[dev];
  return LG_OK;
}

}  // namespace
}  // namespace lg

extern "C" int lg_cgs2_orthogonalize_noalloc(const double* V, int ldv, int n, int ncols, const double* w,
                                             double* r, double* coef, double* norms, void* stream) {
  using namespace lg;
  int rc = cgs2_check_args(V, ldv, n, ncols, w, r, coef, norms);
  if (rc != LG_OK) return rc;
  int grid = cgs2_grid();
  if (grid < 1) {
    g_last_error = "lg_cgs2_orthogonalize_noalloc: no CUDA device";
    return LG_ERR_CUDA;
  }
  if (grid > kNoAllocMaxGrid) grid = kNoAllocMaxGrid;   // more SMs than the array was sized for: use fewer CTAs
  if (cgs2_workspace_doubles(grid) + ST_WORDS > kNoAllocDoubles) {
    g_last_error = "lg_cgs2_orthogonalize_noalloc: workspace exceeds the fixed 0.5 MiB array";
    return LG_ERR_INVALID;
  }
  double* ws = nullptr;
  rc = scratch_address(&ws);
  if (rc != LG_OK) return rc;
  // cgs2_run clears the status words (cudaMemsetAsync, no allocation) before
  // the passes; partial sums and scalars are written before they are read.
  return cgs2_run(V, ldv, n, ncols, w, r, coef, norms, static_cast<cudaStream_t>(stream), grid, ws,
                  reinterpret_cast<int*>(ws + cgs2_workspace_doubles(grid)));
}
