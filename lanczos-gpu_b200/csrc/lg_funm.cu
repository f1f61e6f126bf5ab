// lg_funm.cu — f(A) v and v^T f(A) v by m-step Lanczos quadrature on the
// eigsh engine (no restart), f in {log, exp, sqrt, inv}.
//
// Reference: python/gpu_eigsh/_cuda_funm.cu:40-251 (compute_funm_apply,
// compute_funm_qform, compute_funm_debug) with src/matrix_function.cuh:82-274:
// m Lanczos steps with CGS + conditional DGKS that stop cleanly at an
// invariant subspace (no random restart), T_m eigendecomposed by LAPACK dstev
// on the host, f applied to the Ritz values (log needs theta > 0, sqrt
// theta >= 0, inv theta != 0, else status -2), then
//   f(A) v     ~ ||v|| V S f(Theta) S^T e1   (a Dgemv on the device)
//   v^T f(A) v ~ ||v||^2 sum_i S[0, i]^2 f(Theta_i).
//
// Here the Lanczos steps are the plan's fused step kernels (SpMV with the
// normalisation folded in, CGS2 with the DGKS test on the device, one host
// synchronisation at the end), the small side runs in one CTA on the device
// (Sturm bisection + inverse iteration, lg_tridiag.cuh) and produces the
// combination coefficients, and y = V q is the basis kernel's Ritz mode,
// written straight into the caller's numbering.
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_solver.h"
#include "lg_tridiag.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

namespace lg {

namespace {

constexpr int kFunmThreads = 128;   // >= max_ncv

enum { FUNM_OK = 0, FUNM_BAD_FUNC = -1, FUNM_BAD_EIG = -2, FUNM_ZERO = -3, FUNM_TRIDIAG = -4 };

// One CTA: eigenpairs of T (alpha[0..m), beta[1..m) off-diagonal), f(Theta)
// with the reference's domain rules, q = vnorm * S f(Theta) S^T e1 and
// qf = vnorm^2 sum_i S[0, i]^2 f(Theta_i).  status: 0, -2 or -4.
__global__ void __launch_bounds__(kFunmThreads)
funm_small_kernel(const double* __restrict__ alpha, const double* __restrict__ beta, int m, int func, double vnorm,
                  double* __restrict__ Z, double* __restrict__ F, double* __restrict__ q, double* __restrict__ qf,
                  int* __restrict__ status) {
  __shared__ double d[kMaxCols], e[kMaxCols], e2[kMaxCols], th[kMaxCols], fth[kMaxCols], w[kMaxCols];
  __shared__ int cl[kMaxCols];
  __shared__ double onenrm;
  __shared__ int bad;
  const int t = threadIdx.x;
  if (t == 0) bad = 0;
  for (int i = t; i < m; i += kFunmThreads) {
    d[i] = alpha[i];
    e[i] = i + 1 < m ? beta[i + 1] : 0.0;
    e2[i] = e[i] * e[i];
  }
  __syncthreads();
  if (!tridiag_eigen_cta<kFunmThreads>(d, e, e2, m, th, Z, F, cl, &onenrm)) {
    if (t == 0) *status = FUNM_TRIDIAG;
    return;
  }
  for (int i = t; i < m; i += kFunmThreads) {
    const double x = th[i];
    double f = 0.0;
    bool ok = true;
    switch (func) {
      case LG_FUNC_LOG: ok = x > 0.0; f = ok ? log(x) : 0.0; break;
      case LG_FUNC_EXP: f = exp(x); break;
      case LG_FUNC_SQRT: ok = x >= 0.0; f = ok ? sqrt(x) : 0.0; break;
      default: ok = x != 0.0; f = ok ? 1.0 / x : 0.0; break;
    }
    if (!ok) bad = 1;
    fth[i] = f;
    w[i] = Z[(size_t)i * m] * f;   // S[0, i] f(Theta_i)
  }
  __syncthreads();
  if (bad) {
    if (t == 0) *status = FUNM_BAD_EIG;
    return;
  }
  // q[j] = vnorm sum_i S[j, i] S[0, i] f(Theta_i), fixed order in i
  for (int j = t; j < m; j += kFunmThreads) {
    double s = 0.0;
    for (int i = 0; i < m; ++i) s += Z[(size_t)i * m + j] * w[i];
    q[j] = vnorm * s;
  }
  if (t == 0) {
    double s = 0.0;
    for (int i = 0; i < m; ++i) s += Z[(size_t)i * m] * w[i];
    *qf = vnorm * vnorm * s;
    *status = FUNM_OK;
  }
}

__global__ void gather_perm_funm_kernel(double* __restrict__ out, const double* __restrict__ in,
                                        const int* __restrict__ perm, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = in[perm[i]];
}

}  // namespace

#define LG_TRY(expr)                                                                          \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      g_last_error = std::string("CUDA error ") + cudaGetErrorString(_e) + " in funm";        \
      return (_e == cudaErrorMemoryAllocation) ? LG_ERR_NOMEM : LG_ERR_CUDA;                  \
    }                                                                                         \
  } while (0)

// m Lanczos steps from v (no restart; stop at an invariant subspace).  On
// success *m_actual is the depth reached (0 for a zero v) and *vnorm = ||v||;
// the basis is V[:, 0..m_actual), alpha/beta hold T.
int Solver::funm_factor(const double* v, int io_on_device, int m, int* m_actual, double* vnorm) {
  if (comm) {
    g_last_error = "funm is not available with a row-partitioned plan";
    return LG_ERR_INVALID;
  }
  if (m < 1 || m > max_ncv || m > n || !v) {
    g_last_error = "funm: need 1 <= m <= min(n, max_ncv) and a vector";
    return LG_ERR_INVALID;
  }
  std::memset(&opts, 0, sizeof(opts));
  launches = 0;
  ktimes.clear();
  ev_used = 0;
  LG_TRY(cudaMemsetAsync(state, 0, sizeof(int) * ST_WORDS, stream));
  LG_TRY(cudaMemsetAsync(scal, 0, sizeof(double) * SC_WORDS, stream));
  LG_TRY(cudaMemsetAsync(alpha, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(beta, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(V, 0, sizeof(double) * vsize(), stream));
  LG_TRY(cudaMemsetAsync(R, 0, sizeof(double) * (size_t)ld, stream));
  const cudaMemcpyKind kind = io_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (d_perm) {
    LG_TRY(cudaMemcpyAsync(W, v, sizeof(double) * (size_t)n, kind, stream));
    gather_perm_funm_kernel<<<num_sm * 4, 256, 0, stream>>>(R, W, d_perm, n);
    LG_TRY(cudaGetLastError());
  } else {
    LG_TRY(cudaMemcpyAsync(R, v, sizeof(double) * (size_t)n, kind, stream));
  }
  LG_TRY(norm_partials(stream, grid_gs, R, ld, partC));
  nrowsC = grid_gs;
  inC = partC;
  {
    std::vector<double> part((size_t)grid_gs * kPartStride);
    LG_TRY(cudaMemcpyAsync(part.data(), partC, sizeof(double) * part.size(), cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaStreamSynchronize(stream));
    double s = 0.0;
    for (int r = 0; r < grid_gs; ++r) s += part[(size_t)r * kPartStride + kPartScalar];
    *vnorm = std::sqrt(s);
    if (!std::isfinite(s)) {
      g_last_error = "funm: non-finite input vector";
      return LG_ERR_NUMERIC;
    }
    if (s == 0.0) {
      *m_actual = 0;
      return LG_OK;
    }
  }
  int rc = extend(0, m, BETA_INIT);
  if (rc != LG_OK) return rc;
  int depth = m, last_pass3 = -1;
  for (;;) {
    rc = sync_state();
    if (rc != LG_OK) return rc;
    const int status = h_state[ST_STATUS];
    if (status == STATUS_RUNNING) break;
    const int s = h_state[ST_STEP];
    if ((status != STATUS_PASS3 && status != STATUS_BREAKDOWN) || s < 0 || s >= m) {
      g_last_error = "funm: unexpected device status";
      return LG_ERR_NUMERIC;
    }
    rc = clear_status();
    if (rc != LG_OK) return rc;
    if (status == STATUS_PASS3 && s != last_pass3) {
      last_pass3 = s;
      rc = pass3(s);
      if (rc == LG_OK && s + 1 < m) rc = extend(s + 1, m, BETA_STEP);
      if (rc != LG_OK) return rc;
      continue;
    }
    // invariant subspace after step s (or a third pass that did not restore
    // the norm): stop with s + 1 steps, as the reference does
    depth = s + 1;
    break;
  }
  *m_actual = depth;
  return LG_OK;
}

int Solver::funm(const double* v, int io_on_device, int m, int func, int mode, double* y, double* value,
                 int* m_actual) {
  if (func < LG_FUNC_LOG || func > LG_FUNC_INV || (mode != 0 && mode != 1) || (mode == 1 && !y) ||
      (mode == 0 && !value) || !m_actual) {
    g_last_error = "funm: invalid arguments";
    return LG_ERR_INVALID;
  }
  double vnorm = 0.0;
  int ma = 0;
  int rc = funm_factor(v, io_on_device, m, &ma, &vnorm);
  if (rc != LG_OK) return rc;
  *m_actual = ma;
  if (ma == 0) {   // zero vector: y = 0, the reference's status -3
    if (mode == 1) {
      if (io_on_device) LG_TRY(cudaMemsetAsync(y, 0, sizeof(double) * (size_t)n, stream));
      else std::fill(y, y + n, 0.0);
    } else {
      *value = 0.0;
    }
    LG_TRY(cudaStreamSynchronize(stream));
    *m_actual = FUNM_ZERO;
    return LG_OK;
  }
  // small side: Z (m x m), F (inverse-iteration scratch), q, qf, status
  const size_t zdbl = (size_t)kMaxCols * kMaxCols, fdbl = 4 * (size_t)kMaxCols * kFunmThreads;
  if (!funm_ws) LG_TRY(cudaMalloc(&funm_ws, sizeof(double) * (zdbl + fdbl + kMaxCols + 8)));
  double* Z = funm_ws;
  double* F = Z + zdbl;
  double* q = F + fdbl;
  double* qf = q + kMaxCols;
  int* st = reinterpret_cast<int*>(qf + 4);
  funm_small_kernel<<<1, kFunmThreads, 0, stream>>>(alpha, beta, ma, func, vnorm, Z, F, q, qf, st);
  LG_TRY(cudaGetLastError());
  int hst = 0;
  double hqf = 0.0;
  LG_TRY(cudaMemcpyAsync(&hst, st, sizeof(int), cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaMemcpyAsync(&hqf, qf, sizeof(double), cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaStreamSynchronize(stream));
  if (hst != FUNM_OK) {
    *m_actual = hst;   // -2 (f undefined at a Ritz value) or -4 (tridiagonal failure), as the reference
    return LG_OK;
  }
  if (mode == 0) {
    *value = hqf;
    return LG_OK;
  }
  // y = V q in the caller's numbering (basis kernel, Ritz mode, one column)
  double* Y = y;
  if (!io_on_device) {
    if (!Ytmp || ytmp_elems < (size_t)n) {
      if (Ytmp) cudaFree(Ytmp);
      Ytmp = nullptr;
      LG_TRY(cudaMalloc(&Ytmp, sizeof(double) * (size_t)n));
      ytmp_elems = (size_t)n;
    }
    Y = Ytmp;
  }
  BasisArgs ba;
  ba.V = V;
  ba.vl = vl;
  ba.n = n;
  ba.m = ma;
  ba.kq = 1;
  ba.Q = q;
  ba.ldq = ma;
  ba.restart = 0;
  ba.Y = Y;
  ba.ldy = n;
  ba.rowmajor = 0;
  ba.ymap = d_perm;
  ba.state = state;
  LG_TRY(basis_update(basis_plan(n, ma, 1, grid_basis), ba, stream));
  if (!io_on_device) LG_TRY(cudaMemcpyAsync(y, Ytmp, sizeof(double) * (size_t)n, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaStreamSynchronize(stream));
  return LG_OK;
}

// The raw basis (n x m_actual, column-major, caller's numbering), alpha and
// beta (beta[0] = 0, beta[m_actual] = final residual norm) for tests.
int Solver::funm_debug(const double* v, int m, double* V_out, double* alpha_out, double* beta_out, int* m_actual) {
  double vnorm = 0.0;
  int ma = 0;
  int rc = funm_factor(v, 0, m, &ma, &vnorm);
  if (rc != LG_OK) return rc;
  *m_actual = ma;
  if (ma == 0) return LG_OK;
  // V[:, 0..ma) through the basis kernel with Q = I
  std::vector<double> I((size_t)ma * ma, 0.0);
  for (int i = 0; i < ma; ++i) I[(size_t)i * ma + i] = 1.0;
  double* dI = nullptr;
  double* dY = nullptr;
  LG_TRY(cudaMalloc(&dI, sizeof(double) * I.size()));
  cudaError_t e = cudaMalloc(&dY, sizeof(double) * (size_t)n * ma);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dI, I.data(), sizeof(double) * I.size(), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) {
    BasisArgs ba;
    ba.V = V;
    ba.vl = vl;
    ba.n = n;
    ba.m = ma;
    ba.kq = ma;
    ba.Q = dI;
    ba.ldq = ma;
    ba.restart = 0;
    ba.Y = dY;
    ba.ldy = n;
    ba.rowmajor = 0;
    ba.ymap = d_perm;
    ba.state = state;
    e = basis_update(basis_plan(n, ma, ma, grid_basis), ba, stream);
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(V_out, dY, sizeof(double) * (size_t)n * ma, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(alpha_out, alpha, sizeof(double) * ma, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(beta_out, beta, sizeof(double) * ma, cudaMemcpyDeviceToHost, stream);
  std::vector<double> part((size_t)nrowsC * kPartStride);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(part.data(), inC, sizeof(double) * part.size(), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(dI);
  cudaFree(dY);
  LG_TRY(e);
  double s = 0.0;
  for (int r = 0; r < nrowsC; ++r) s += part[(size_t)r * kPartStride + kPartScalar];
  beta_out[0] = 0.0;
  beta_out[ma] = ma < m ? 0.0 : std::sqrt(s);
  return LG_OK;
}

}  // namespace lg
