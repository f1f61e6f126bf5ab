// lg_cg.cu — shift-invert operator: (A - sigma I)^-1 v by conjugate gradients.
//
// Reference: src/inner_solve.cuh:110-200 (cg_solve_shifted: one SpMV, one
// Daxpy for the shift, two blocking Ddot reads and four BLAS-1 calls per
// iteration) and :213-241 (ShiftInvertOperator, which ignores a failed solve).
//
// Here one CG iteration is two kernels and no host round trip:
//   cg_k1: p = r + beta p_old is formed on the fly inside the SpMV gather
//          (double-buffered p, so no CTA overwrites what another gathers),
//          Ap = (A - sigma I) p, and p.Ap reduced by the last CTA to finish;
//   cg_k2: alpha = rr / p.Ap; x += alpha p; r -= alpha Ap; r.r reduced the
//          same way.
// The convergence test ||r|| < cg_tol ||b|| runs on the device at the top of
// cg_k1; once it passes, the remaining queued iterations return at once.  The
// host launches iterations in chunks sized from the previous solve and reads
// a flag word between chunks.  Solves that stop at cg_max_iters are counted
// and reported (LG_ERR_CG_NOCONV) instead of being silently accepted.
#include "lg_common.cuh"
#include "lg_csr.cuh"
#include "lg_kernels.cuh"
#include "lg_solver.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace lg {

namespace {

enum { CG_RR = 0 /* two slots: 0, 1 */, CG_PAP = 2, CG_TOL2 = 3, CG_SCAL_WORDS = 8 };
enum { CGF_DONE = 0, CGF_ITERS = 1, CG_FLAG_WORDS = 4 };
// CGF_DONE: 0 running, 1 converged, 2 iteration limit, 3 breakdown (p.Ap ~ 0)

// Block total -> per-block slot; the last CTA to arrive sums the slots in a
// fixed order and writes *out.  No waiting: the other CTAs just exit.
__device__ void lastblock_sum(double block_total, double* part, unsigned* counter, double* out,
                              double* extra_out = nullptr, double extra_scale = 0.0) {
  __shared__ int am_last;
  if (threadIdx.x == 0) {
    part[blockIdx.x] = block_total;
    __threadfence();
    const unsigned prev = atomicAdd(counter, 1u);
    am_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!am_last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    double s = 0.0;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += 32) s += __ldcg(part + i);
    s = warp_sum(s);
    if (threadIdx.x == 0) {
      *out = s;
      if (extra_out) *extra_out = extra_scale * s;
      *counter = 0u;
    }
  }
}

__global__ void __launch_bounds__(256)
cg_init_kernel(int n, const double* __restrict__ b, double* __restrict__ x, double* __restrict__ r,
               double* __restrict__ pa, double* __restrict__ pb, double tol, double* cg_scal, double* part,
               unsigned* counter) {
  __shared__ double scr[32];
  double acc = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double bi = b[i];
    x[i] = 0.0;
    r[i] = bi;
    pa[i] = 0.0;
    pb[i] = 0.0;
    acc += bi * bi;
  }
  acc = block_sum(acc, scr);
  lastblock_sum(acc, part, counter, &cg_scal[CG_RR], &cg_scal[CG_TOL2], tol * tol);
}

template <typename VT, int L>
__global__ void __launch_bounds__(256)
cg_k1_kernel(int n, const int* __restrict__ rowptr, const int* __restrict__ col, const VT* __restrict__ val,
             double sigma, const double* __restrict__ r, const double* __restrict__ p_old,
             double* __restrict__ p_new, double* __restrict__ Ap, int it, int maxit, double* cg_scal,
             double* part, unsigned* counter, int* flags, const int* state) {
  if (flags[CGF_DONE] != 0 || state[ST_STATUS] != STATUS_RUNNING) return;
  __shared__ double scr[32];
  double beta = 0.0;
  if (it > 0) {
    const double rr = cg_scal[CG_RR + (it & 1)];
    const double rrp = cg_scal[CG_RR + ((it - 1) & 1)];
    int done = 0;
    if (rr < cg_scal[CG_TOL2]) done = 1;
    else if (it >= maxit) done = 2;
    if (done) {
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        flags[CGF_ITERS] = it;
        flags[CGF_DONE] = done;
      }
      return;
    }
    beta = rr / rrp;
  }
  // Each lane group works on two rows at once so that the dependent load
  // chains (row_ptr -> col -> r, p gathers) of the two rows overlap.
  const int lane = threadIdx.x & (L - 1);
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  const int rows_per_warp = 32 / L;
  double local = 0.0;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; (long long)w * rows_per_warp * 2 < n;
       w += warps_total) {
    const int rowA = w * rows_per_warp * 2 + ((threadIdx.x & 31) / L);
    const int rowB = rowA + rows_per_warp;
    const bool okA = rowA < n, okB = rowB < n;
    int kA = 0, eA = 0, kB = 0, eB = 0;
    if (okA) { kA = __ldg(rowptr + rowA) + lane; eA = __ldg(rowptr + rowA + 1); }
    if (okB) { kB = __ldg(rowptr + rowB) + lane; eB = __ldg(rowptr + rowB + 1); }
    double accA = 0.0, accB = 0.0;
    while (kA < eA || kB < eB) {
      if (kA < eA) {
        const int c = __ldg(col + kA);
        accA += (double)__ldg(val + kA) * (r[c] + beta * p_old[c]);
      }
      if (kB < eB) {
        const int c = __ldg(col + kB);
        accB += (double)__ldg(val + kB) * (r[c] + beta * p_old[c]);
      }
      kA += L;
      kB += L;
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) {
      accA += __shfl_xor_sync(0xffffffffu, accA, o);
      accB += __shfl_xor_sync(0xffffffffu, accB, o);
    }
    if (lane == 0) {
      if (okA) {
        const double pn = r[rowA] + beta * p_old[rowA];
        const double ap = accA - sigma * pn;
        p_new[rowA] = pn;
        Ap[rowA] = ap;
        local += pn * ap;
      }
      if (okB) {
        const double pn = r[rowB] + beta * p_old[rowB];
        const double ap = accB - sigma * pn;
        p_new[rowB] = pn;
        Ap[rowB] = ap;
        local += pn * ap;
      }
    }
  }
  local = block_sum(local, scr);
  lastblock_sum(local, part, counter, &cg_scal[CG_PAP]);
}

__global__ void __launch_bounds__(256)
cg_k2_kernel(int n, double* __restrict__ x, double* __restrict__ r, const double* __restrict__ p,
             const double* __restrict__ Ap, int it, double* cg_scal, double* part, unsigned* counter, int* flags,
             const int* state) {
  if (flags[CGF_DONE] != 0 || state[ST_STATUS] != STATUS_RUNNING) return;
  __shared__ double scr[32];
  const double pAp = cg_scal[CG_PAP];
  if (!(fabs(pAp) >= kSafeMin)) {   // also catches NaN
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      flags[CGF_ITERS] = it + 1;
      flags[CGF_DONE] = 3;
    }
    return;
  }
  const double a = cg_scal[CG_RR + (it & 1)] / pAp;
  double local = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    x[i] += a * p[i];
    const double ri = r[i] - a * Ap[i];
    r[i] = ri;
    local += ri * ri;
  }
  local = block_sum(local, scr);
  lastblock_sum(local, part, counter, &cg_scal[CG_RR + ((it + 1) & 1)]);
}

template <typename VT>
cudaError_t launch_k1(const CsrDev& A, const VT* val, cudaStream_t st, int grid, double sigma, const double* r,
                      const double* p_old, double* p_new, double* Ap, int it, int maxit, double* cg_scal,
                      double* part, unsigned* counter, int* flags, const int* state) {
#define LG_K1(LN)                                                                                        \
  cg_k1_kernel<VT, LN><<<grid, 256, 0, st>>>(A.n, A.rowptr, A.col, val, sigma, r, p_old, p_new, Ap, it, maxit, \
                                             cg_scal, part, counter, flags, state)
  switch (A.lanes) {
    case 2: LG_K1(2); break;
    case 4: LG_K1(4); break;
    case 8: LG_K1(8); break;
    case 16: LG_K1(16); break;
    default: LG_K1(32); break;
  }
#undef LG_K1
  return cudaGetLastError();
}

}  // namespace

#define LG_TRY(expr)                                                                              \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess) {                                                                      \
      g_last_error = std::string("CUDA error ") + cudaGetErrorString(_e) + " in shift-invert";     \
      return (_e == cudaErrorMemoryAllocation) ? LG_ERR_NOMEM : LG_ERR_CUDA;                      \
    }                                                                                             \
  } while (0)

int Solver::prepare_shift_invert() {
  if (!cg_ws) {
    LG_TRY(cudaMalloc(&cg_ws, sizeof(double) * (size_t)ld * 5));
    LG_TRY(cudaMemsetAsync(cg_ws, 0, sizeof(double) * (size_t)ld * 5, stream));
    cg_grid = num_sm * 8;   // 8 CTAs of 256 threads: every SM at full thread occupancy
    LG_TRY(cudaMalloc(&cg_part, sizeof(double) * (size_t)cg_grid));
    LG_TRY(cudaMalloc(&cg_scal, sizeof(double) * CG_SCAL_WORDS));
    LG_TRY(cudaMalloc(&cg_counter, sizeof(unsigned)));
    LG_TRY(cudaMemsetAsync(cg_counter, 0, sizeof(unsigned), stream));
    LG_TRY(cudaMalloc(&cg_flags, sizeof(int) * CG_FLAG_WORDS));
    LG_TRY(cudaMallocHost(&h_cg_flags, sizeof(int) * (CG_FLAG_WORDS + 2)));
  }
  cg_chunk = 64;
  return LG_OK;
}

int Solver::cg_solve(const double* b, double* x) {
  double* r = cg_ws;
  double* pbuf[2] = {cg_ws + ld, cg_ws + 2 * (size_t)ld};
  double* Ap = cg_ws + 3 * (size_t)ld;
  const int maxit = opts.cg_max_iters > 0 ? opts.cg_max_iters : (n > 214748364 ? 2147483647 : 10 * n);
  const double tol = opts.cg_tol > 0.0 ? opts.cg_tol : 1e-12;
  LG_TRY(cudaMemsetAsync(cg_flags, 0, sizeof(int) * CG_FLAG_WORDS, stream));
  ++launches;
  cg_init_kernel<<<cg_grid, 256, 0, stream>>>(n, b, x, r, pbuf[0], pbuf[1], tol, cg_scal, cg_part, cg_counter);
  LG_TRY(cudaGetLastError());
  int it = 0;
  int chunk = cg_chunk;
  for (;;) {
    const int it_end = std::min(it + chunk, maxit + 1);
    // per iteration: CSR + gathers of r, p (once) + p, Ap written; then
    // x, p, Ap, r read and x, r written
    const double it_bytes = ((A.val32 ? 8.0 : 12.0) * (double)nnz + 4.0 * (n + 1) + 32.0 * n) + 48.0 * n;
    for (; it < it_end; ++it) {
      double* pn = pbuf[it & 1];
      const double* po = pbuf[(it + 1) & 1];
      LG_TRY(timed(LG_K_CG, it_bytes, it < maxit ? 2 : 1, [&]() -> cudaError_t {
        cudaError_t e;
        if (A.val32)
          e = launch_k1<float>(A, A.val32, stream, cg_grid, opts.sigma, r, po, pn, Ap, it, maxit, cg_scal,
                               cg_part, cg_counter, cg_flags, state);
        else
          e = launch_k1<double>(A, A.val64, stream, cg_grid, opts.sigma, r, po, pn, Ap, it, maxit, cg_scal,
                                cg_part, cg_counter, cg_flags, state);
        if (e != cudaSuccess || it >= maxit) return e;
        cg_k2_kernel<<<cg_grid, 256, 0, stream>>>(n, x, r, pn, Ap, it, cg_scal, cg_part, cg_counter, cg_flags,
                                                   state);
        return cudaGetLastError();
      }));
    }
    LG_TRY(cudaMemcpyAsync(h_cg_flags, cg_flags, sizeof(int) * CG_FLAG_WORDS, cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaMemcpyAsync(h_cg_flags + CG_FLAG_WORDS, state, sizeof(int), cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaStreamSynchronize(stream));
    if (h_cg_flags[CG_FLAG_WORDS] != STATUS_RUNNING) return LG_OK;  // step was stopped upstream
    if (h_cg_flags[CGF_DONE] != 0) break;
    if (it > maxit) break;
    chunk = std::max(16, chunk / 2);
  }
  const int iters = h_cg_flags[CGF_ITERS];
  cg_iters += iters;
  if (h_cg_flags[CGF_DONE] != 1) ++cg_failures;
  // next solve: queue about as many iterations as this one needed
  cg_chunk = std::max(16, iters + 8);
  return LG_OK;
}

int Solver::apply_shift_invert(int j, int beta_mode) {
  double* Vj = V + vidx(vl, 0, j);       // column j of the basis
  double* b = cg_ws + 4 * (size_t)ld;    // the same vector, contiguous (CG right-hand side)
  LG_TRY(timed(LG_K_OTHER, 24.0 * n, 1, [&] {
    return normalize_step(stream, num_sm * 8, n, R, Vj, (int)vl.rs, b, partC, nrowsC, j, beta_mode, alpha, beta, scal,
                          state);
  }));
  return cg_solve(b, W);
}

}  // namespace lg
