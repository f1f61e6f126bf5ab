// lg_imgp.cu — the graphbandwidth-dependent symmetric-normalised graph
// Laplacian of the IMGP precision operator, and its derivative, in CSR order.
//
// Reference: _build_laplacian_cache (python/gpu_eigsh/imgp.py:142-189).  With
// w_e = exp(-d2_e / (4 k^2)) per edge e = (s, d):
//   du_i   = [self_loops] + sum_{e at i} w_e
//   adj_e  = w_e / (du_s du_d)
//   deg_i  = [self_loops] du_i^-2 + sum_{e at i} adj_e
//   L_ii   = (1 - du_i^-2 / deg_i) / k^2        (self_loops; else 1 / k^2)
//   L_sd   = -adj_e / sqrt(deg_s deg_d) / k^2
// The reference forms the sums with scatter_add over the edge list; here every
// sum is a row sum of the CSR that stores each edge in both directions, so it
// is one thread per row, without atomics, in a fixed order.  dL/dk follows by
// the chain rule through the same three passes (dw/dk = w d2 / (2 k^3)); the
// SLQ backward uses it in place of autograd through the cache.
//
// Three kernels: (1) du, du'; (2) deg, deg' (gathers du of the neighbours);
// (3) the off-diagonal values and the diagonal with their derivatives.
// Arithmetic is fp64; values are stored in the operator's element type.
#include "lg_common.cuh"

#include "../../include/lanczos_b200.h"

#include <string>

namespace lg {
extern thread_local std::string g_last_error;

namespace {

constexpr int kLapThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kLapThreads)
lap_degree_kernel(int n, const int* __restrict__ rowptr, const T* __restrict__ d2, double inv4k2, double dscale,
                  double base, double* __restrict__ du, double* __restrict__ ddu) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    double s = base, ds = 0.0;
    for (int k = rowptr[i]; k < rowptr[i + 1]; ++k) {
      const double q = (double)d2[k];
      const double w = exp(-q * inv4k2);
      s += w;
      ds += w * q * dscale;
    }
    du[i] = s;
    ddu[i] = ds;
  }
}

template <typename T>
__global__ void __launch_bounds__(kLapThreads)
lap_norm_kernel(int n, const int* __restrict__ rowptr, const int* __restrict__ col, const T* __restrict__ d2,
                double inv4k2, double dscale, int self_loops, const double* __restrict__ du,
                const double* __restrict__ ddu, double* __restrict__ deg, double* __restrict__ ddeg) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const double ui = du[i], dui = ddu[i];
    double s = 0.0, ds = 0.0;
    if (self_loops) {
      s = 1.0 / (ui * ui);
      ds = -2.0 * dui / (ui * ui * ui);
    }
    for (int k = rowptr[i]; k < rowptr[i + 1]; ++k) {
      const int jn = col[k];
      const double uj = du[jn], duj = ddu[jn];
      const double q = (double)d2[k];
      const double w = exp(-q * inv4k2), dw = w * q * dscale;
      const double a = w / (ui * uj);
      s += a;
      ds += dw / (ui * uj) - a * (dui / ui + duj / uj);
    }
    deg[i] = s;
    ddeg[i] = ds;
  }
}

template <typename T>
__global__ void __launch_bounds__(kLapThreads)
lap_values_kernel(int n, const int* __restrict__ rowptr, const int* __restrict__ col, const T* __restrict__ d2,
                  double inv4k2, double dscale, double ik2, double ik3, int self_loops, const double* __restrict__ du,
                  const double* __restrict__ ddu, const double* __restrict__ deg, const double* __restrict__ ddeg,
                  T* __restrict__ offval, T* __restrict__ diag, T* __restrict__ doffval, T* __restrict__ ddiag) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const double ui = du[i], dui = ddu[i], gi = deg[i], dgi = ddeg[i];
    for (int k = rowptr[i]; k < rowptr[i + 1]; ++k) {
      const int jn = col[k];
      const double uj = du[jn], duj = ddu[jn], gj = deg[jn], dgj = ddeg[jn];
      const double q = (double)d2[k];
      const double w = exp(-q * inv4k2), dw = w * q * dscale;
      const double a = w / (ui * uj);
      const double da = dw / (ui * uj) - a * (dui / ui + duj / uj);
      const double rs = 1.0 / sqrt(gi * gj);
      const double t = a * rs * ik2;
      const double dt = da * rs * ik2 - t * 0.5 * (dgi / gi + dgj / gj) - 2.0 * t * ik3 / ik2;
      offval[k] = (T)(-t);
      if (doffval) doffval[k] = (T)(-dt);
    }
    double dv, ddv;
    if (self_loops) {
      const double g = 1.0 / (ui * ui * gi);
      const double dg = -2.0 * dui / (ui * ui * ui * gi) - dgi / (ui * ui * gi * gi);
      dv = (1.0 - g) * ik2;
      ddv = -dg * ik2 - 2.0 * (1.0 - g) * ik3;
    } else {
      dv = ik2;
      ddv = -2.0 * ik3;
    }
    diag[i] = (T)dv;
    if (ddiag) ddiag[i] = (T)ddv;
  }
}

template <typename T>
cudaError_t laplacian_t(int n, const int* rowptr, const int* col, const T* d2, double kappa, int self_loops,
                        T* offval, T* diag, T* doffval, T* ddiag, double* work, cudaStream_t st) {
  const double k2 = kappa * kappa;
  const double inv4k2 = 1.0 / (4.0 * k2);
  const double dscale = 1.0 / (2.0 * k2 * kappa);     // dw/dk = w * d2 / (2 k^3)
  const double ik2 = 1.0 / k2, ik3 = 1.0 / (k2 * kappa);
  double* du = work;
  double* ddu = work + n;
  double* deg = work + 2 * (size_t)n;
  double* ddeg = work + 3 * (size_t)n;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long need = ((long long)n + kLapThreads - 1) / kLapThreads;
  const int grid = (int)(need < 8LL * sms ? need : 8LL * sms);
  lap_degree_kernel<T><<<grid, kLapThreads, 0, st>>>(n, rowptr, d2, inv4k2, dscale, self_loops ? 1.0 : 0.0, du, ddu);
  lap_norm_kernel<T><<<grid, kLapThreads, 0, st>>>(n, rowptr, col, d2, inv4k2, dscale, self_loops, du, ddu, deg, ddeg);
  lap_values_kernel<T><<<grid, kLapThreads, 0, st>>>(n, rowptr, col, d2, inv4k2, dscale, ik2, ik3, self_loops, du, ddu,
                                                     deg, ddeg, offval, diag, doffval, ddiag);
  return cudaGetLastError();
}

}  // namespace
}  // namespace lg

using namespace lg;

extern "C" int lg_imgp_laplacian(int n, long long nnz, const int* rowptr, const int* col, int dtype, const void* d2,
                                 double graphbandwidth, int self_loops, void* offval, void* diag, void* doffval,
                                 void* ddiag, double* work, void* stream) {
  if (n < 1 || nnz < 0 || nnz > 2147483647LL || !rowptr || (nnz > 0 && (!col || !d2 || !offval)) || !diag || !work ||
      (dtype != LG_F32 && dtype != LG_F64) || !(graphbandwidth != 0.0)) {
    g_last_error = "lg_imgp_laplacian: invalid arguments";
    return LG_ERR_INVALID;
  }
  if ((doffval == nullptr) != (ddiag == nullptr)) {
    g_last_error = "lg_imgp_laplacian: doffval and ddiag go together";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == LG_F64)
    e = laplacian_t<double>(n, rowptr, col, static_cast<const double*>(d2), graphbandwidth, self_loops,
                            static_cast<double*>(offval), static_cast<double*>(diag), static_cast<double*>(doffval),
                            static_cast<double*>(ddiag), work, st);
  else
    e = laplacian_t<float>(n, rowptr, col, static_cast<const float*>(d2), graphbandwidth, self_loops,
                           static_cast<float*>(offval), static_cast<float*>(diag), static_cast<float*>(doffval),
                           static_cast<float*>(ddiag), work, st);
  if (e != cudaSuccess) {
    g_last_error = std::string("lg_imgp_laplacian: ") + cudaGetErrorString(e);
    return LG_ERR_CUDA;
  }
  return LG_OK;
}
