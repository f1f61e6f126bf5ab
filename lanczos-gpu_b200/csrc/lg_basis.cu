// lg_basis.cu — dense basis contraction  out = V[:, 0:m] * Q[:, 0:kq].
//
// Two uses:
//  * implicit restart (reference src/irlm_lanczos.cu:299-338: Dgemm V*Q into a
//    second n x ncv buffer, D2D copy back, Dscal/Daxpy for the residual,
//    Dnrm2).  Here the update is done in place, one row tile at a time: the
//    tile of V is staged in shared memory by TMA, contracted with Q (kept in
//    shared memory), written back over the same rows, and the restart
//    residual r <- rcoef * r + tau * (V Q)[:, kq-1] plus its norm partials are
//    produced in the same pass.  V is read once and written once.
//  * Ritz vectors (reference src/lanczos_ops.cuh:318-338, Dgemm V*S then a
//    D2H copy) written straight into the caller's layout (column-major or
//    row-major n x k), so no host transpose is needed.
//
// The contraction is FP64.  Arithmetic intensity is ~2*kq/8 flop/byte
// (~4-8 at the configurations of interest), i.e. at the HBM/FP64 ridge.
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_tma.cuh"

namespace lg {

namespace {
constexpr int kBsThreads = 512;
constexpr int kBsMaxOut = 16;    // outputs per thread: kq <= 8 * 16 = 128

struct BsSmem {
  static constexpr int kBars = 0;
  static constexpr int kFlag = 64;
  static constexpr int kScr = 128;                // 32 doubles
  static constexpr int kQ = kScr + 32 * 8;        // m * kq doubles, then stages
};
}  // namespace

static size_t basis_smem_bytes(int S, int T, int m, int kq) {
  size_t q = (size_t)m * kq * sizeof(double);
  q = (q + 127) / 128 * 128;
  return (size_t)BsSmem::kQ + q + (size_t)S * m * T * sizeof(double);
}

BasisPlan basis_plan(int ld, int m, int kq, int grid, size_t budget) {
  BasisPlan p;
  p.T = 64;
  size_t fixed = basis_smem_bytes(0, 64, m, kq);
  size_t per = (size_t)m * 64 * sizeof(double);
  int S = (int)((budget - fixed) / per);
  if (S > kMaxStages) S = kMaxStages;
  if (S < 1) S = 1;
  p.S = S;
  p.ntiles = ld / p.T;
  p.grid = grid < p.ntiles ? grid : p.ntiles;
  p.smem = basis_smem_bytes(S, p.T, m, kq);
  return p;
}

__global__ void __launch_bounds__(kBsThreads, 1)
basis_kernel(BasisArgs a, int T, int S, int ntiles) {
  int* state = a.state;
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BsSmem::kBars);
  int* flag = reinterpret_cast<int*>(smem + BsSmem::kFlag);
  double* scr = reinterpret_cast<double*>(smem + BsSmem::kScr);
  double* Qs = reinterpret_cast<double*>(smem + BsSmem::kQ);
  size_t qbytes = ((size_t)a.m * a.kq * sizeof(double) + 127) / 128 * 128;
  double* buf = reinterpret_cast<double*>(smem + BsSmem::kQ + qbytes);

  const int t = threadIdx.x, warp = t >> 5;
  const int m = a.m, kq = a.kq;

  TileRing ring{bars, buf, S, T, m, a.ld, a.V, nullptr};
  ring.init_barriers();

  const int tb = (int)(((long long)ntiles * blockIdx.x) / gridDim.x);
  const int te = (int)(((long long)ntiles * (blockIdx.x + 1)) / gridDim.x);
  const int nt = te - tb;
  if (warp == 0)
    for (int s = 0; s < S && s < nt; ++s) ring.issue(tb + s, s);

  // Q[:, 0:kq] into shared memory, column-major with leading dim m.
  for (int i = t; i < m * kq; i += kBsThreads) {
    const int r = i % m, c = i / m;
    Qs[i] = a.Q[r + (size_t)c * a.ldq];
  }
  __syncthreads();

  double rcoef = 0.0, tau = 0.0;
  if (a.restart) {
    rcoef = a.scal[SC_RCOEF];
    tau = a.scal[SC_TAU];
  }

  const int KG = kBsThreads / T;          // output groups
  const int row = t & (T - 1), kg = t / T;
  double nrm = 0.0;

  for (int it = 0; it < nt; ++it) {
    const int s = it % S;
    if (!ring.wait(s, (uint32_t)((it / S) & 1), flag, state, 200)) {
      ring.drain(it, nt);
      return;
    }
    const double* Vs = ring.stage_ptr(s);
    const size_t grow = (size_t)(tb + it) * T + row;

    double acc[kBsMaxOut];
#pragma unroll
    for (int i = 0; i < kBsMaxOut; ++i) acc[i] = 0.0;
    for (int c = 0; c < m; ++c) {
      const double v = Vs[(size_t)c * T + row];
      const double* qrow = Qs + c;
#pragma unroll
      for (int i = 0; i < kBsMaxOut; ++i) {
        const int k = kg + KG * i;
        if (k < kq) acc[i] += v * qrow[(size_t)k * m];
      }
    }
    // Every thread of this tile has finished reading the stage only after
    // the barrier below; writes go to global memory, so they may happen now.
    if (a.restart) {
#pragma unroll
      for (int i = 0; i < kBsMaxOut; ++i) {
        const int k = kg + KG * i;
        if (k < kq - 1) a.V[grow + (size_t)k * a.ld] = acc[i];
        else if (k == kq - 1) {
          const double r = rcoef * a.R[grow] + tau * acc[i];
          a.R[grow] = r;
          nrm += r * r;
        }
      }
    } else if (grow < (size_t)a.nrows) {
#pragma unroll
      for (int i = 0; i < kBsMaxOut; ++i) {
        const int k = kg + KG * i;
        if (k < kq) {
          if (a.rowmajor) a.Y[grow * (size_t)kq + k] = acc[i];
          else a.Y[grow + (size_t)k * a.ldy] = acc[i];
        }
      }
    }
    __syncthreads();
    if (warp == 0 && it + S < nt) ring.issue(tb + it + S, s);
  }

  if (a.restart) {
    const double tot = block_sum(nrm, scr);
    if (t == 0) a.part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = tot;
  }
}

cudaError_t basis_update(const BasisPlan& p, const BasisArgs& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(basis_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  basis_kernel<<<p.grid, kBsThreads, p.smem, st>>>(a, p.T, p.S, p.ntiles);
  return cudaGetLastError();
}

}  // namespace lg
