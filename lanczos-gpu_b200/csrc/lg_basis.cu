// lg_basis.cu — dense basis contraction  out = V[:, 0:m] * Q[:, 0:kq]  on the
// FP64 tensor cores.
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
// The contraction uses the FP64 MMA instruction (mma.sync m8n8k4 .f64;
// tcgen05 has no f64 kind): each warp owns 8 basis rows of the 64-row tile
// and all ceil(kq/8) output blocks, walking k = 0..m in steps of 4.  Shared
// strides are chosen = 4 (mod 16) doubles so fragment loads are conflict free.
#include "lg_common.cuh"
#include "lg_kernels.cuh"

namespace lg {

namespace {
constexpr int kBsThreads = 256;
constexpr int kTR = 64;                      // basis rows per tile (8 warps x 8 rows)
constexpr int kMaxOB = kMaxCols / 8;         // output blocks of 8 columns

__host__ __device__ inline int pad_stride(int x) {   // x multiple of 4 -> stride = 4 or 12 (mod 16)
  return (x % 16 == 0 || x % 16 == 8) ? x + 4 : x;
}

struct BsGeom {
  int mp, kqp, sv, sq;   // padded k, padded outputs, row stride of the V tile, column stride of Q
  __host__ __device__ BsGeom(int m, int kq) {
    mp = (m + 3) & ~3;
    kqp = (kq + 7) & ~7;
    sv = pad_stride(mp > kqp ? mp : kqp);
    sq = pad_stride(mp);
  }
  __host__ __device__ size_t smem_doubles() const { return (size_t)kqp * sq + (size_t)kTR * sv; }
};

__device__ __forceinline__ void dmma(double& c0, double& c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}
}  // namespace

BasisPlan basis_plan(int n, int m, int kq, int grid) {
  BasisPlan p;
  p.TR = kTR;
  const int ntiles = (n + kTR - 1) / kTR;
  p.grid = grid < ntiles ? grid : ntiles;
  p.smem = BsGeom(m, kq).smem_doubles() * sizeof(double);
  return p;
}

template <int NOB>
__global__ void __launch_bounds__(kBsThreads)
basis_kernel(BasisArgs a) {
  int* state = a.state;
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(16) double sm[];
  __shared__ double scr[32];
  const int m = a.m, kq = a.kq, n = a.n;
  const VLayout vl = a.vl;
  const BsGeom g(m, kq);
  double* Qs = sm;                              // kqp columns x sq (column-major, zero padded)
  double* Vs = sm + (size_t)g.kqp * g.sq;       // kTR rows x sv (row-major, zero padded)
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int gid = lane >> 2, tig = lane & 3;

  for (int i = t; i < g.kqp * g.sq; i += kBsThreads) {
    const int c = i / g.sq, r = i % g.sq;
    Qs[i] = (c < kq && r < m) ? a.Q[r + (size_t)c * a.ldq] : 0.0;
  }
  double rcoef = 0.0, tau = 0.0;
  if (a.restart) {
    rcoef = a.scal[SC_RCOEF];
    tau = a.scal[SC_TAU];
  }
  double nrm = 0.0;
  const int ntiles = (n + kTR - 1) / kTR;
  const int nob = g.kqp / 8;

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row0 = (long long)tile * kTR;
    __syncthreads();   // previous tile consumed; Qs ready on the first pass
    // eight columns of a row at a time (one panel row of the solver's basis:
    // 64 contiguous bytes; consecutive threads take consecutive rows)
    for (int i = t; i < kTR * (g.mp >> 2); i += kBsThreads) {
      const int rr = i % kTR, c = (i / kTR) * 4;
      const long long row = row0 + rr;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        Vs[rr * g.sv + c + q] = (row < n && c + q < m) ? a.V[vidx(vl, row, c + q)] : 0.0;
    }
    __syncthreads();
    double acc[NOB][2];
#pragma unroll
    for (int ob = 0; ob < NOB; ++ob) acc[ob][0] = acc[ob][1] = 0.0;
    const double* arow = Vs + (warp * 8 + gid) * g.sv + tig;
    const double* bcol = Qs + gid * g.sq + tig;
    for (int k0 = 0; k0 < g.mp; k0 += 4) {
      const double av = arow[k0];
#pragma unroll
      for (int ob = 0; ob < NOB; ++ob)
        if (ob < nob) dmma(acc[ob][0], acc[ob][1], av, bcol[ob * 8 * g.sq + k0]);
    }
    __syncthreads();   // all fragment reads of Vs done
#pragma unroll
    for (int ob = 0; ob < NOB; ++ob)
      if (ob < nob) {
        double* o = Vs + (warp * 8 + gid) * g.sv + ob * 8 + 2 * tig;
        o[0] = acc[ob][0];
        o[1] = acc[ob][1];
      }
    __syncthreads();
    if (a.restart) {
      const int kv = kq - 1;   // columns written back into V
      for (int i = t; i < kTR * kv; i += kBsThreads) {
        const int rr = i / kv, k = i % kv;
        const long long row = row0 + rr;
        if (row < n) a.V[vidx(vl, row, k)] = Vs[rr * g.sv + k];
      }
      if (t < kTR) {
        const long long row = row0 + t;
        if (row < n) {
          const double rn = rcoef * a.R[row] + tau * Vs[t * g.sv + kv];
          a.R[row] = rn;
          nrm += rn * rn;
        }
      }
    } else if (a.rowmajor) {
      for (int i = t; i < kTR * kq; i += kBsThreads) {
        const int rr = i / kq, k = i % kq;
        const long long row = row0 + rr;
        if (row < n) a.Y[(a.ymap ? (long long)a.ymap[row] : row) * kq + k] = Vs[rr * g.sv + k];
      }
    } else {
      for (int i = t; i < kTR * kq; i += kBsThreads) {
        const int k = i / kTR, rr = i % kTR;
        const long long row = row0 + rr;
        if (row < n) a.Y[(a.ymap ? (long long)a.ymap[row] : row) + (long long)k * a.ldy] = Vs[rr * g.sv + k];
      }
    }
  }
  if (a.restart) {
    const double tot = block_sum(nrm, scr);
    if (t == 0) a.part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = tot;
  }
}

cudaError_t basis_update(const BasisPlan& p, const BasisArgs& a, cudaStream_t st) {
  const int nob = ((a.kq + 7) & ~7) / 8;
#define LG_BS(N)                                                                                     \
  do {                                                                                               \
    cudaError_t e = cudaFuncSetAttribute(basis_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         (int)p.smem);                                               \
    if (e != cudaSuccess) return e;                                                                  \
    basis_kernel<N><<<p.grid, kBsThreads, p.smem, st>>>(a);                                          \
  } while (0)
  if (nob <= 4) LG_BS(4);
  else if (nob <= 8) LG_BS(8);
  else LG_BS(kMaxOB);
#undef LG_BS
  return cudaGetLastError();
}

}  // namespace lg
