// lg_basis.cu — dense basis contraction  out = V[:, 0:m] * Q[:, 0:kq].
//
// Two uses:
//  * implicit restart (reference src/irlm_lanczos.cu:299-338: Dgemm V*Q into a
//    second n x ncv buffer, D2D copy back, Dscal/Daxpy for the residual,
//    Dnrm2).  Here the update is done in place, one tile of basis rows at a
//    time: the rows (contiguous in the row-major basis) are staged in shared
//    memory with coalesced loads, contracted with Q (kept in shared memory),
//    written back over the same rows, and the restart residual
//    r <- rcoef * r + tau * (V Q)[:, kq-1] plus its norm partials come out of
//    the same pass.  V is read once and written once.
//  * Ritz vectors (reference src/lanczos_ops.cuh:318-338, Dgemm V*S then a
//    D2H copy) written straight into the caller's layout (column-major or
//    row-major n x k), so no host transpose is needed.
//
// FP64 throughout; arithmetic intensity ~kq/4 flop/byte, near the HBM/FP64
// ridge at the configurations of interest.
#include "lg_common.cuh"
#include "lg_kernels.cuh"

namespace lg {

namespace {
constexpr int kBsThreads = 256;
constexpr int kTR = 32;                 // basis rows per tile
constexpr int kKG = kBsThreads / kTR;   // output-column groups
constexpr int kMaxOut = 16;             // kq <= kKG * kMaxOut = 128

__host__ __device__ inline int odd_stride(int m) { return m | 1; }
}  // namespace

static size_t basis_smem(int m, int kq) {
  return ((size_t)m * kq + (size_t)kTR * odd_stride(m > kq ? m : kq)) * sizeof(double);
}

BasisPlan basis_plan(int n, int m, int kq, int grid) {
  BasisPlan p;
  p.TR = kTR;
  const int ntiles = (n + kTR - 1) / kTR;
  p.grid = grid < ntiles ? grid : ntiles;
  p.smem = basis_smem(m, kq);
  return p;
}

__global__ void __launch_bounds__(kBsThreads)
basis_kernel(BasisArgs a) {
  int* state = a.state;
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(16) double sm[];
  __shared__ double scr[32];
  const int m = a.m, kq = a.kq, n = a.n, ldv = a.ldv;
  const int MS = odd_stride(m > kq ? m : kq);
  double* Qs = sm;                      // m x kq, column-major (leading dim m)
  double* Vs = sm + (size_t)m * kq;     // kTR x MS
  const int t = threadIdx.x;

  for (int i = t; i < m * kq; i += kBsThreads) {
    const int r = i % m, c = i / m;
    Qs[i] = a.Q[r + (size_t)c * a.ldq];
  }
  double rcoef = 0.0, tau = 0.0;
  if (a.restart) {
    rcoef = a.scal[SC_RCOEF];
    tau = a.scal[SC_TAU];
  }
  const int r = t & (kTR - 1), kg = t / kTR;
  double nrm = 0.0;
  const int ntiles = (n + kTR - 1) / kTR;

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row0 = (long long)tile * kTR;
    __syncthreads();   // previous tile fully consumed (and Qs ready on the first pass)
    for (int i = t; i < kTR * m; i += kBsThreads) {
      const int rr = i / m, c = i % m;
      const long long row = row0 + rr;
      Vs[rr * MS + c] = (row < n) ? a.V[row * ldv + c] : 0.0;
    }
    __syncthreads();
    double acc[kMaxOut];
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) acc[i] = 0.0;
    const double* vrow = Vs + r * MS;
    for (int c = 0; c < m; ++c) {
      const double v = vrow[c];
#pragma unroll
      for (int i = 0; i < kMaxOut; ++i) {
        const int k = kg + kKG * i;
        if (k < kq) acc[i] += v * Qs[c + (size_t)k * m];
      }
    }
    __syncthreads();   // all reads of Vs done
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
      const int k = kg + kKG * i;
      if (k < kq) Vs[r * MS + k] = acc[i];
    }
    __syncthreads();
    if (a.restart) {
      const int kv = kq - 1;   // columns written back into V
      for (int i = t; i < kTR * kv; i += kBsThreads) {
        const int rr = i / kv, k = i % kv;
        const long long row = row0 + rr;
        if (row < n) a.V[row * ldv + k] = Vs[rr * MS + k];
      }
      if (t < kTR) {
        const long long row = row0 + t;
        if (row < n) {
          const double rn = rcoef * a.R[row] + tau * Vs[t * MS + kv];
          a.R[row] = rn;
          nrm += rn * rn;
        }
      }
    } else if (a.rowmajor) {
      for (int i = t; i < kTR * kq; i += kBsThreads) {
        const int rr = i / kq, k = i % kq;
        const long long row = row0 + rr;
        if (row < n) a.Y[row * kq + k] = Vs[rr * MS + k];
      }
    } else {
      for (int i = t; i < kTR * kq; i += kBsThreads) {
        const int k = i / kTR, rr = i % kTR;
        const long long row = row0 + rr;
        if (row < n) a.Y[row + (long long)k * a.ldy] = Vs[rr * MS + k];
      }
    }
  }
  if (a.restart) {
    const double tot = block_sum(nrm, scr);
    if (t == 0) a.part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = tot;
  }
}

cudaError_t basis_update(const BasisPlan& p, const BasisArgs& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(basis_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  basis_kernel<<<p.grid, kBsThreads, p.smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lg
