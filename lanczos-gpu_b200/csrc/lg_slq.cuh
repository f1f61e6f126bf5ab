// lg_slq.cuh — building blocks shared by the SLQ kernels (lg_slq.cu: the fused
// sparse-operator engine; lg_slq_block.cu: block kernels around a caller's
// matvec).
//
// Block layout: every block of probe vectors is n x ld, row-major, ld even;
// columns [0, B) are active (B <= 128).  When B is odd, column B is padding:
// loads treat it as zero and stores write zero there.  One warp owns one row
// at a time; lane l owns columns 2l, 2l+1 of each 64-column chunk, so a row
// is one coalesced 256-byte (fp32) / 512-byte (fp64) access per chunk.
//
// Column reductions (dots and norms over the n rows, per probe column): each
// CTA sums its warps into one partial row, and the last CTA to finish (an
// atomic ticket, no waiting) reduces the partial rows in a fixed order into
// `out`, so every result is bitwise repeatable.  The next kernel on the
// stream reads `out`.
#pragma once

#include "lg_common.cuh"

namespace lg {
namespace slq {

constexpr int kT = 512;                    // threads per CTA
constexpr int kW = kT / 32;                // warps per CTA
constexpr int kMaxB = 128;                 // active columns per block
constexpr int kQ = 4;                      // column-sum quantities per partial row
constexpr int kRowStride = kQ * kMaxB;     // doubles per partial row
constexpr int kQT = 128;                   // threads of the per-probe small-side kernel
constexpr unsigned kFull = 0xffffffffu;

template <typename T> struct Vec2;
template <> struct Vec2<float> { using type = float2; };
template <> struct Vec2<double> { using type = double2; };

// Pair load of columns c0, c0+1; the second is zero when it is padding.
template <typename T>
__device__ __forceinline__ void ld2m(const T* p, bool second, double& x, double& y) {
  const auto v = *reinterpret_cast<const typename Vec2<T>::type*>(p);
  x = (double)v.x;
  y = second ? (double)v.y : 0.0;
}
template <typename T>
__device__ __forceinline__ void ld2m_cs(const T* p, bool second, double& x, double& y) {
  const auto v = __ldcs(reinterpret_cast<const typename Vec2<T>::type*>(p));
  x = (double)v.x;
  y = second ? (double)v.y : 0.0;
}
template <typename T>
__device__ __forceinline__ void st2(T* p, double x, double y) {
  typename Vec2<T>::type v;
  v.x = (T)x;
  v.y = (T)y;
  *reinterpret_cast<typename Vec2<T>::type*>(p) = v;
}
// Value as stored in a block of element type T.
template <typename T>
__device__ __forceinline__ double rnd(double x) {
  return (double)(T)x;
}

struct ColSum {
  double* part;        // gridDim.x rows of kRowStride doubles
  double* out;         // kRowStride doubles: out[q * kMaxB + c]
  unsigned* counter;   // zero between kernels
};

// acc[q][ch][i]: this lane's sum of quantity q for column ch*64 + 2*lane + i
// over the rows it visited.  Called by every thread of the CTA, once, at the
// end of the kernel.
template <int NCH>
__device__ void colsum_finish(const double (&acc)[kQ][NCH][2], int nq, int B, const ColSum cs) {
  __shared__ double s_w[kW * kMaxB];
  __shared__ bool s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = threadIdx.x;
  for (int q = 0; q < nq; ++q) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = ch * 64 + 2 * lane;
      if (c0 < B) {
        s_w[warp * kMaxB + c0] = acc[q][ch][0];
        s_w[warp * kMaxB + c0 + 1] = acc[q][ch][1];
      }
    }
    __syncthreads();
    for (int c = t; c < B; c += kT) {
      double s = 0.0;
      for (int w = 0; w < kW; ++w) s += s_w[w * kMaxB + c];
      cs.part[(size_t)blockIdx.x * kRowStride + q * kMaxB + c] = s;
    }
    __syncthreads();
  }
  __threadfence();
  if (t == 0) s_last = (atomicAdd(cs.counter, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int E = nq * B, R = gridDim.x;
  const int G = max(1, kT / E);
  if (t < G * E) {
    const int e = t % E, g = t / E;
    const int off = (e / B) * kMaxB + (e % B);
    const double* p = cs.part + off;
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    int r = g;
    for (; r + 3 * G < R; r += 4 * G) {
      s0 += __ldcg(p + (size_t)r * kRowStride);
      s1 += __ldcg(p + (size_t)(r + G) * kRowStride);
      s2 += __ldcg(p + (size_t)(r + 2 * G) * kRowStride);
      s3 += __ldcg(p + (size_t)(r + 3 * G) * kRowStride);
    }
    for (; r < R; r += G) s0 += __ldcg(p + (size_t)r * kRowStride);
    s_w[g * E + e] = (s0 + s1) + (s2 + s3);
  }
  __syncthreads();
  if (t < E) {
    double s = 0.0;
    for (int g = 0; g < G; ++g) s += s_w[g * E + t];
    cs.out[(t / B) * kMaxB + (t % B)] = s;
  }
  if (t == 0) *cs.counter = 0u;
}

// Sparse symmetric operator A = shift I + L, L = diag + off-diagonal CSR.
struct Op {
  int n;
  const int* rowptr;
  const int* col;
  double shift;
};

// y += sum_k off[k] X[col[k], :] over row `row` (and yk with doff when DERIV),
// for this lane's columns.  The warp loads 32 (col, value) pairs at once and
// broadcasts them by shuffle, so the row gathers issue back to back.
template <typename T, int NCH, bool DERIV>
__device__ __forceinline__ void gather_row(const Op& op, const T* __restrict__ off, const T* __restrict__ doff,
                                           const T* __restrict__ X, int ld, int B, long long row, int lane,
                                           double (&y)[NCH][2], double (&yk)[NCH][2]) {
  const int kb = __ldg(op.rowptr + row), ke = __ldg(op.rowptr + row + 1);
  for (int k0 = kb; k0 < ke; k0 += 32) {
    const int kk = k0 + lane;
    int ci = 0;
    double av = 0.0, dv = 0.0;
    if (kk < ke) {
      ci = __ldg(op.col + kk);
      av = (double)__ldg(off + kk);
      if (DERIV) dv = (double)__ldg(doff + kk);
    }
    const int cnt = min(32, ke - k0);
#pragma unroll 8
    for (int s = 0; s < cnt; ++s) {
      const long long c = __shfl_sync(kFull, ci, s);
      const double a = __shfl_sync(kFull, av, s);
      const double d = DERIV ? __shfl_sync(kFull, dv, s) : 0.0;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int c0 = ch * 64 + 2 * lane;
        if (c0 < B) {
          double vx, vy;
          ld2m(X + c * ld + c0, c0 + 1 < B, vx, vy);
          y[ch][0] += a * vx;
          y[ch][1] += a * vy;
          if (DERIV) {
            yk[ch][0] += d * vx;
            yk[ch][1] += d * vy;
          }
        }
      }
    }
  }
}

// Grid used by every SLQ kernel (partial rows are indexed by blockIdx.x).
int slq_grid();

}  // namespace slq
}  // namespace lg
