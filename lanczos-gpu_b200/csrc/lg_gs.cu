// lg_gs.cu — classical Gram-Schmidt passes against the Lanczos basis V.
//
// One Lanczos step j (reference: src/irlm_lanczos.cu:110-148 with
// cgs_orthogonalize / dgks_reorth, src/lanczos_ops.cuh:113-192) is split into
//
//   spmv   : w = A v_j                                   (lg_spmv.cu)
//   pass 1 : h = V^T w,  ||w||^2                         gs_project
//   pass 2 : r1 = w - V h, then s = V^T r1, ||r1||^2     gs_correct_project
//   pass 3 : r2 = r1 - V s, ||r2||^2, alpha_j = h_j+s_j  gs_correct
//
// so V (n x (j+1), column-major, leading dimension ld) is streamed three
// times per step instead of four (cuBLAS Dgemv T/N twice in the reference).
// Pass 2 needs every V element twice (row dot for r1, column dot for s); the
// row tile therefore lives in shared memory, brought in by TMA bulk copies
// (cp.async.bulk, one per column segment) through an S-stage mbarrier ring.
//
// Each CTA owns a contiguous range of row tiles and writes one row of
// partial sums; the consumer of those partials (the next kernel) reduces them
// in a fixed order in every CTA, so results are bitwise repeatable and no
// atomics or grid-wide spin waits are involved.
#include "lg_common.cuh"
#include "lg_kernels.cuh"
#include "lg_tma.cuh"

namespace lg {

// Reduce `nrows` partial rows: columns [0, nc) into out[0..nc), the scalar
// slot into *scal_out.  Every thread of the block gets the same values.
__device__ void reduce_partials(const double* __restrict__ part, int nrows, int nc,
                                double* out, double* scal_out, double* red /* >= 512 doubles */) {
  const int t = threadIdx.x;
  const int slot = t & 127, grp = t >> 7;   // 4 row groups of 128 column slots
  double acc = 0.0;
  if (slot < nc) {
    int r = grp;
#pragma unroll 4
    for (; r < nrows; r += 4) acc += part[(size_t)r * kPartStride + slot];
  }
  red[grp * 128 + slot] = acc;
  // scalar column: warp 0
  double sc = 0.0;
  if (t < 32) {
    for (int r = t; r < nrows; r += 32) sc += part[(size_t)r * kPartStride + kPartScalar];
    sc = warp_sum(sc);
  }
  __syncthreads();
  if (t < nc) out[t] = red[t] + red[128 + t] + red[256 + t] + red[384 + t];
  if (t == 0) *scal_out = sc;
  __syncthreads();
}


// Shared-memory layout of the three pass kernels.
struct GsSmem {
  static constexpr int kBars = 0;                       // 8 mbarriers (64 B)
  static constexpr int kFlag = 64;                      // int flag
  static constexpr int kCoef = 128;                     // 128 doubles
  static constexpr int kRed = kCoef + 128 * 8;          // 512 doubles
  static constexpr int kRvec = kRed + 512 * 8;          // 256 doubles
  static constexpr int kScr = kRvec + 256 * 8;          // 32 doubles
  static constexpr int kBuf = kScr + 32 * 8;            // stages (16-byte aligned)
};

size_t gs_smem_bytes(int S, int T, int ncols) {
  return (size_t)GsSmem::kBuf + (size_t)S * (ncols + 1) * T * sizeof(double);
}

// MODE 1: project   (vec = W or R)           -> part_out: V^T vec, ||vec||^2
// MODE 2: correct+project (vec = W)          -> R = vec - V coef ; part_out: V^T R, ||R||^2
// MODE 3: correct   (vec = R)                -> R = vec - V coef ; part_out: ||R||^2
template <int MODE>
__global__ void __launch_bounds__(kGsThreads, 1)
gs_pass_kernel(const double* __restrict__ V, int ld, int ncols, int T, int S, int ntiles,
               const double* vec, double* Rout, const double* __restrict__ part_in, int nrows_in,
               double* __restrict__ part_out, double* scal, double* alpha, int j, int alpha_mode,
               int* state) {
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GsSmem::kBars);
  int* flag = reinterpret_cast<int*>(smem + GsSmem::kFlag);
  double* coef = reinterpret_cast<double*>(smem + GsSmem::kCoef);
  double* red = reinterpret_cast<double*>(smem + GsSmem::kRed);
  double* rvec = reinterpret_cast<double*>(smem + GsSmem::kRvec);
  double* scr = reinterpret_cast<double*>(smem + GsSmem::kScr);
  double* buf = reinterpret_cast<double*>(smem + GsSmem::kBuf);

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  TileRing ring{bars, buf, S, T, ncols, ld, V, vec};
  ring.init_barriers();

  // Tile range of this CTA.
  const int tb = (int)(((long long)ntiles * blockIdx.x) / gridDim.x);
  const int te = (int)(((long long)ntiles * (blockIdx.x + 1)) / gridDim.x);
  const int nt = te - tb;

  // Start streaming before the (latency-bound) reduction of the inputs.
  if (warp == 0)
    for (int s = 0; s < S && s < nt; ++s) ring.issue(tb + s, s);

  if (MODE != 1) {
    double sc;
    reduce_partials(part_in, nrows_in, ncols, coef, &sc, red);
    if (blockIdx.x == 0 && t == 0) {
      if (MODE == 2) {
        scal[SC_WN2] = sc;
        scal[SC_HJ] = coef[ncols - 1];
      } else {
        scal[SC_R1N2] = sc;
        if (alpha_mode == 1) alpha[j] = scal[SC_HJ] + coef[j];
        else if (alpha_mode == 2) alpha[j] += coef[j];
      }
    }
  }

  double acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.0;
  double nrm = 0.0;

  const int TPR = kGsThreads / T;         // threads per row in the row-dot phase
  const int row = t & (T - 1), part = t / T;

  for (int it = 0; it < nt; ++it) {
    const int s = it % S;
    if (!ring.wait(s, (uint32_t)((it / S) & 1), flag, state, 100 + MODE)) {
      ring.drain(it, nt);
      return;
    }
    const double* Vs = ring.stage_ptr(s);
    const double* xs = Vs + (size_t)ncols * T;    // the vector segment
    const size_t grow = (size_t)(tb + it) * T;

    const double* colsrc = xs;                    // vector used by the column dots
    if (MODE != 1) {
      // row dots: y[row] = x[row] - sum_c V[row, c] * coef[c]
      double p = 0.0;
      for (int c = part; c < ncols; c += TPR) p += Vs[(size_t)c * T + row] * coef[c];
      red[part * T + row] = p;
      __syncthreads();
      if (t < T) {
        double y = xs[t];
        for (int q = 0; q < TPR; ++q) y -= red[q * T + t];
        rvec[t] = y;
        Rout[grow + t] = y;
        nrm += y * y;
      }
      __syncthreads();
      colsrc = rvec;
    } else {
      if (t < T) nrm += xs[t] * xs[t];
    }
    if (MODE != 3) {
      // column dots: acc[c] += sum_row V[row, c] * colsrc[row]
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int c = warp + 16 * k;
        if (c < ncols) {
          const double* vc = Vs + (size_t)c * T;
          double a = 0.0;
          for (int r = lane; r < T; r += 32) a += vc[r] * colsrc[r];
          acc[k] += a;
        }
      }
    }
    __syncthreads();
    if (warp == 0 && it + S < nt) ring.issue(tb + it + S, s);
  }

  double* prow = part_out + (size_t)blockIdx.x * kPartStride;
  if (MODE != 3) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = warp + 16 * k;
      if (c < ncols) {
        const double v = warp_sum(acc[k]);
        if (lane == 0) prow[c] = v;
      }
    }
  }
  const double tot = block_sum(nrm, scr);
  if (t == 0) prow[kPartScalar] = tot;
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
static int pick_stages(int T, int ncols, size_t budget) {
  const size_t per = (size_t)(ncols + 1) * T * sizeof(double);
  size_t s = (budget - GsSmem::kBuf) / per;
  if (s > (size_t)kMaxStages) s = kMaxStages;
  return (int)s;
}

GsPlan gs_plan(int ld, int ncols, int grid, size_t smem_budget) {
  GsPlan p;
  // Larger row tiles when few columns are live keep each stage >= ~16 KB.
  int T = 64;
  if ((ncols + 1) * 64 * 8 < 16384 && ld % 128 == 0) T = 128;
  if ((ncols + 1) * 128 * 8 < 16384 && ld % 256 == 0) T = 256;
  int S = pick_stages(T, ncols, smem_budget);
  while (S < 2 && T > 64) { T >>= 1; S = pick_stages(T, ncols, smem_budget); }
  if (S < 1) S = 1;
  p.T = T;
  p.S = S;
  p.ntiles = ld / T;
  p.grid = grid < p.ntiles ? grid : p.ntiles;
  p.smem = gs_smem_bytes(S, T, ncols);
  return p;
}

template <int MODE>
static cudaError_t launch_gs(const GsPlan& p, cudaStream_t st, const double* V, int ld, int ncols,
                             const double* vec, double* Rout, const double* part_in, int nrows_in,
                             double* part_out, double* scal, double* alpha, int j, int alpha_mode,
                             int* state) {
  auto kern = gs_pass_kernel<MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  kern<<<p.grid, kGsThreads, p.smem, st>>>(V, ld, ncols, p.T, p.S, p.ntiles, vec, Rout, part_in, nrows_in,
                                           part_out, scal, alpha, j, alpha_mode, state);
  return cudaGetLastError();
}

cudaError_t gs_project(const GsPlan& p, cudaStream_t st, const double* V, int ld, int ncols,
                       const double* vec, double* part_out, int* state) {
  return launch_gs<1>(p, st, V, ld, ncols, vec, nullptr, nullptr, 0, part_out, nullptr, nullptr, 0, 0,
                      state);
}

cudaError_t gs_correct_project(const GsPlan& p, cudaStream_t st, const double* V, int ld, int ncols,
                               const double* W, double* R, const double* part_in, int nrows_in,
                               double* part_out, double* scal, int* state) {
  return launch_gs<2>(p, st, V, ld, ncols, W, R, part_in, nrows_in, part_out, scal, nullptr, 0, 0, state);
}

cudaError_t gs_correct(const GsPlan& p, cudaStream_t st, const double* V, int ld, int ncols, double* R,
                       const double* part_in, int nrows_in, double* part_out, double* scal, double* alpha,
                       int j, int alpha_mode, int* state) {
  return launch_gs<3>(p, st, V, ld, ncols, R, R, part_in, nrows_in, part_out, scal, alpha, j, alpha_mode,
                      state);
}

}  // namespace lg
