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

#include <algorithm>

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

// 16-byte asynchronous copy global -> shared; `bytes` < 16 zero-fills the rest
__device__ __forceinline__ void bs_cp16(void* smem, const void* gmem, int bytes) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bs_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bs_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
}  // namespace

template <int NOB>
__global__ void basis_kernel(BasisArgs a);

// CTAs of basis_kernel<NOB> resident on one SM with `smem` bytes of dynamic
// shared memory (0 when unknown).
static int basis_resident(int nob, size_t smem) {
  int res = 0;
  cudaError_t e = cudaSuccess;
  if (nob <= 4) e = cudaFuncSetAttribute(basis_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  else if (nob <= 8) e = cudaFuncSetAttribute(basis_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  else e = cudaFuncSetAttribute(basis_kernel<kMaxOB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    if (nob <= 4) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, basis_kernel<4>, kBsThreads, smem);
    else if (nob <= 8) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, basis_kernel<8>, kBsThreads, smem);
    else e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, basis_kernel<kMaxOB>, kBsThreads, smem);
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return res;
}

BasisPlan basis_plan(int n, int m, int kq, int grid) {
  BasisPlan p;
  p.TR = kTR;
  const int ntiles = (n + kTR - 1) / kTR;
  p.grid = grid < ntiles ? grid : ntiles;
  const BsGeom g(m, kq);
  // One tile buffer per CTA: the copies of one CTA overlap the MMAs of the
  // other CTAs on the SM, and the shared memory of a second buffer would halve
  // the resident CTAs.  Measured against two buffers per CTA: V*Q per
  // configuration-1 solve (m = 60) 2.03 -> 1.96 ms, per R-MAT solve (m = 96,
  // one CTA per SM with two buffers, two with one) 212 -> 133 ms.
  // At m = 127: Q 128 x 132 and one 64 x 132 tile, 203 KB.
  p.smem = g.smem_doubles() * sizeof(double);
  // one wave: the tiles are dealt to the CTAs in a grid-strided loop, every
  // CTA the same count, so CTAs beyond the resident ones would only form a
  // second wave as long as the first
  int dev = 0, nsm = 0;
  const int res = basis_resident(g.kqp / 8, p.smem);
  if (res > 0 && cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && nsm > 0)
    p.grid = std::max(1, std::min(p.grid, nsm * res));
  (void)cudaGetLastError();
  return p;
}

// One tile of kTR basis rows: out = V[rows, 0:m] Q[0:m, 0:kq] on the FP64
// tensor cores.  The tile's rows of V arrive in shared memory by asynchronous
// 16-byte copies, two columns at a time (in the solver's panel layout the 64
// rows of a panel are 4 KB of contiguous memory); the next tile's copies start
// once this one is contracted and written, and the other CTAs of the SM keep
// the memory busy meanwhile.
// Register caps: four CTAs of 256 threads per SM for the narrow instantiation
// (up to 32 outputs: the restart of ncv <= 64), two for the wider ones.
template <int NOB>
__global__ void __launch_bounds__(kBsThreads, NOB <= 4 ? 4 : 2)
basis_kernel(BasisArgs a) {
  int* state = a.state;
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(16) double sm[];
  __shared__ double scr[32];
  __shared__ double kvcol[kTR];   // restart: column kq - 1 of the tile's product
  const int m = a.m, kq = a.kq, n = a.n;
  const VLayout vl = a.vl;
  const BsGeom g(m, kq);
  double* Qs = sm;                              // kqp columns x sq (column-major, zero padded)
  double* Vs = sm + (size_t)g.kqp * g.sq;       // one tile of kTR rows x sv
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
  const int npanels = (g.mp + 7) / 8;

  // copies of one tile: index i -> (panel, row, pair of columns), consecutive
  // threads on consecutive pairs of a panel row, then the next rows
  auto issue = [&](int tile, double* buf) {
    const long long row0 = (long long)tile * kTR;
    for (int i = t; i < kTR * npanels * 4; i += kBsThreads) {
      const int c = (i / (kTR * 4)) * 8 + 2 * (i & 3);
      const int rr = (i >> 2) % kTR;
      if (c >= g.mp) continue;
      const long long row = row0 + rr;
      const int bytes = (row < n && c < m) ? (c + 1 < m ? 16 : 8) : 0;
      bs_cp16(buf + rr * g.sv + c, bytes ? a.V + vidx(vl, row, c) : a.V, bytes);
    }
  };

  if ((int)blockIdx.x < ntiles) issue(blockIdx.x, Vs);
  bs_commit();
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row0 = (long long)tile * kTR;
    const int next = tile + gridDim.x;
    bs_wait<0>();
    __syncthreads();   // every thread's copies (and Qs on the first pass)
    // two accumulator sets (k steps alternate between them) halve the chain
    // of dependent MMAs; they are added once at the end
    double acc[NOB][2], acc2[NOB][2];
#pragma unroll
    for (int ob = 0; ob < NOB; ++ob) acc[ob][0] = acc[ob][1] = acc2[ob][0] = acc2[ob][1] = 0.0;
    const double* arow = Vs + (warp * 8 + gid) * g.sv + tig;
    const double* bcol = Qs + gid * g.sq + tig;
    int k0 = 0;
    constexpr bool kSplit = NOB <= 8;   // the widest tiles keep one set (registers)
    for (; kSplit && k0 + 4 < g.mp; k0 += 8) {
      const double av = arow[k0], av2 = arow[k0 + 4];
#pragma unroll
      for (int ob = 0; ob < NOB; ++ob)
        if (ob < nob) {
          dmma(acc[ob][0], acc[ob][1], av, bcol[ob * 8 * g.sq + k0]);
          dmma(acc2[ob][0], acc2[ob][1], av2, bcol[ob * 8 * g.sq + k0 + 4]);
        }
    }
    for (; k0 < g.mp; k0 += 4) {
      const double av = arow[k0];
#pragma unroll
      for (int ob = 0; ob < NOB; ++ob)
        if (ob < nob) dmma(acc[ob][0], acc[ob][1], av, bcol[ob * 8 * g.sq + k0]);
    }
#pragma unroll
    for (int ob = 0; ob < NOB; ++ob) {
      acc[ob][0] += acc2[ob][0];
      acc[ob][1] += acc2[ob][1];
    }
    if (kSplit && a.restart) {
      // straight from the fragments into V (the tile's rows of V are all in
      // Vs already): a thread holds columns ob*8 + 2*tig, +1 of one row, and
      // the 32 lanes of a warp cover 8 rows x 64 contiguous bytes per panel
      const int kv = kq - 1;
      const int rr = warp * 8 + gid;
      const long long row = row0 + rr;
#pragma unroll
      for (int ob = 0; ob < NOB; ++ob)
        if (ob < nob) {
          const int c = ob * 8 + 2 * tig;
          if (row < n) {
            double* dst = a.V + vidx(vl, row, c);
            if (c + 1 < kv) *reinterpret_cast<double2*>(dst) = make_double2(acc[ob][0], acc[ob][1]);
            else if (c < kv) dst[0] = acc[ob][0];
          }
          if (c == kv) kvcol[rr] = acc[ob][0];
          if (c + 1 == kv) kvcol[rr] = acc[ob][1];
        }
      __syncthreads();   // kvcol complete; every fragment read of Vs done
      if (t < kTR) {
        const long long r = row0 + t;
        if (r < n) {
          const double rn = rcoef * a.R[r] + tau * kvcol[t];
          a.R[r] = rn;
          nrm += rn * rn;
        }
      }
      if (next < ntiles) {
        issue(next, Vs);
        bs_commit();
      }
      continue;
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
      const int kv = kq - 1;   // columns written back into V, panel by panel (64 contiguous bytes per row)
      const int kpan = (kv + 7) / 8;
      for (int i = t; i < kTR * kpan * 8; i += kBsThreads) {
        const int c = (i / (kTR * 8)) * 8 + (i & 7);
        const int rr = (i >> 3) % kTR;
        const long long row = row0 + rr;
        if (row < n && c < kv) a.V[vidx(vl, row, c)] = Vs[rr * g.sv + c];
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
    __syncthreads();   // the outputs are read out of Vs before Vs receives copies again
    if (next < ntiles) {
      issue(next, Vs);
      bs_commit();
    }
  }
  bs_wait<0>();
  if (a.restart) {
    const double tot = block_sum(nrm, scr);
    if (t == 0) a.part_out[(size_t)blockIdx.x * kPartStride + kPartScalar] = tot;
  }
}

cudaError_t basis_update(const BasisPlan& p, const BasisArgs& a_in, cudaStream_t st) {
  BasisArgs a = a_in;
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
