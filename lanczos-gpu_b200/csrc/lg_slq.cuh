// lg_slq.cuh — building blocks shared by the SLQ kernels (lg_slq.cu).
//
// Block layout: every block of probe vectors is n x ld, row-major; columns
// [0, B) are active (B <= 128) and columns [B, ld) are padding, read as zero
// and written as zero.  ld is a multiple of 4 (fp32) or 2 (fp64) so that a
// lane's vector of VEC = 16 / sizeof(T) elements is one aligned 16-byte load.
//
// Lane layout <T, LPR>: a group of LPR lanes owns one row (RPW = 32 / LPR rows
// per warp); lane l of the group owns columns ch * LPR * VEC + l * VEC + v.
// For 64 fp32 probes LPR = 16: a half-warp reads a 256-byte row with one
// float4 per lane, and every gather instruction of the warp fetches two
// neighbour rows.  The streaming kernels (recurrence, lambda, xi, norms) use
// the same layout.
//
// Column reductions (dots and norms over the n rows, per probe column): the
// row groups of a warp are combined by shuffles, the warps of a CTA in shared
// memory into one partial row, and the last CTA to finish (an atomic ticket,
// no waiting) reduces the partial rows in a fixed order into `out`, so every
// result is bitwise repeatable.  The next kernel on the stream reads `out`.
#pragma once

#include "lg_common.cuh"

namespace lg {
namespace slq {

constexpr int kT = 512;                    // threads per CTA
constexpr int kW = kT / 32;                // warps per CTA
constexpr int kMinCta = 3;                 // CTAs per SM the kernels are built for
constexpr int kMaxB = 128;                 // active columns per block
constexpr int kQ = 4;                      // column-sum quantities per partial row
constexpr int kRowStride = kQ * kMaxB;     // doubles per partial row
constexpr int kQT = 128;                   // threads of the per-probe small-side kernel
constexpr unsigned kFull = 0xffffffffu;

template <typename T, int N> struct VecT;
template <> struct VecT<float, 2> { using type = float2; };
template <> struct VecT<float, 4> { using type = float4; };
template <> struct VecT<double, 2> { using type = double2; };

template <typename T> struct Lanes { static constexpr int VEC = 16 / (int)sizeof(T); };

// Vector load of N consecutive elements (aligned); elements at or beyond
// `valid` read as zero.
template <typename T, int N>
__device__ __forceinline__ void ldvec(const T* p, int valid, T (&v)[N]) {
  const auto x = *reinterpret_cast<const typename VecT<T, N>::type*>(p);
  const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = (i < valid) ? e[i] : T(0);
}
template <typename T, int N>
__device__ __forceinline__ void ldvecd(const T* p, int valid, double (&v)[N]) {
  T t[N];
  ldvec<T, N>(p, valid, t);
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = (double)t[i];
}
template <typename T, int N>
__device__ __forceinline__ void stvec(T* p, const double (&v)[N], int valid) {
  typename VecT<T, N>::type x;
  T* e = reinterpret_cast<T*>(&x);
#pragma unroll
  for (int i = 0; i < N; ++i) e[i] = (i < valid) ? (T)v[i] : T(0);
  *reinterpret_cast<typename VecT<T, N>::type*>(p) = x;
}

template <typename T, int N>
__device__ __forceinline__ void stvec_t(T* p, const T (&v)[N], int valid) {
  typename VecT<T, N>::type x;
  T* e = reinterpret_cast<T*>(&x);
#pragma unroll
  for (int i = 0; i < N; ++i) e[i] = (i < valid) ? v[i] : T(0);
  *reinterpret_cast<typename VecT<T, N>::type*>(p) = x;
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

// acc[q][ch][v] (q < NQ): this lane's sum of quantity q for its column
// ch * LPR * VEC + (lane % LPR) * VEC + v over the rows it visited.  Called by
// every thread of the CTA, once, at the end of the kernel.
template <int NQ, int VEC, int NCH, int LPR>
__device__ void colsum_finish(double (&acc)[NQ][NCH][VEC], int B, const ColSum cs) {
  static_assert(NQ >= 1 && NQ <= kQ, "at most kQ quantities per partial row");
  constexpr int nq = NQ;
  __shared__ double s_w[kW * kMaxB];
  __shared__ bool s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = threadIdx.x;
  const int l = lane % LPR;
  for (int q = 0; q < nq; ++q) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        double s = acc[q][ch][v];
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) s += __shfl_xor_sync(kFull, s, o);
        const int c = ch * LPR * VEC + l * VEC + v;
        if (lane < LPR && c < B) s_w[warp * kMaxB + c] = s;
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

// Row-group geometry of a lane in layout <T, LPR>.
template <typename T, int LPR>
struct RowLanes {
  static constexpr int VEC = Lanes<T>::VEC;
  static constexpr int RPW = 32 / LPR;
  static constexpr int CPP = LPR * VEC;      // columns per pass
  int lane, l, sub;
  __device__ RowLanes() : lane(threadIdx.x & 31), l((threadIdx.x & 31) % LPR), sub((threadIdx.x & 31) / LPR) {}
  __device__ int col0(int ch) const { return ch * CPP + l * VEC; }
  __device__ long long first_row() const { return ((long long)blockIdx.x * kW + (threadIdx.x >> 5)) * RPW + sub; }
  __device__ long long first_warp_row() const { return ((long long)blockIdx.x * kW + (threadIdx.x >> 5)) * RPW; }
  __device__ static long long stride() { return (long long)gridDim.x * kW * RPW; }
};

// y += sum_k off[k] X[col[k], :] over the row of this lane group (and yk with
// doff when DERIV), accumulated in T.  The group loads LPR * U (col, value)
// pairs at once (U per lane) and broadcasts them by shuffle; the loop runs to
// the longest row of the warp so that every lane takes part in every shuffle.
// Narrow rows (LPR < 8 lanes: blocks of few probes) take U = 8 / LPR pairs per
// lane, so that eight neighbour rows are gathered per trip instead of LPR;
// the neighbours are still added in index order.
template <typename T, int LPR, int NCH, bool DERIV>
__device__ __forceinline__ void gather_rows(const Op& op, const T* __restrict__ off, const T* __restrict__ doff,
                                            const T* __restrict__ X, int ld, int B, bool valid, long long row,
                                            const RowLanes<T, LPR>& g, T (&y)[NCH][Lanes<T>::VEC],
                                            T (&yk)[NCH][Lanes<T>::VEC]) {
  constexpr int VEC = Lanes<T>::VEC;
  constexpr int U = LPR >= 8 ? 1 : 8 / LPR;
  const int kb = valid ? __ldg(op.rowptr + row) : 0;
  const int cnt = valid ? __ldg(op.rowptr + row + 1) - kb : 0;
  int mx = cnt;
#pragma unroll
  for (int o = LPR; o < 32; o <<= 1) mx = max(mx, __shfl_xor_sync(kFull, mx, o));
  const int base = g.lane - g.l;
  auto add = [&](long long c, T a, T d) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 < B) {
        // padding columns (>= B) of X may hold anything: they only ever
        // reach the padding columns of y, which are neither stored nor summed
        T v[VEC];
        ldvec<T, VEC>(X + c * ld + c0, VEC, v);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          y[ch][i] += a * v[i];
          if (DERIV) yk[ch][i] += d * v[i];
        }
      }
    }
  };
  if constexpr (U == 1) {
    for (int k0 = 0; k0 < mx; k0 += LPR) {
      const int kk = k0 + g.l;
      int ci = 0;
      T av = T(0), dv = T(0);
      if (kk < cnt) {
        ci = __ldg(op.col + kb + kk);
        av = __ldg(off + kb + kk);
        if (DERIV) dv = __ldg(doff + kb + kk);
      }
      const int nb = min(LPR, mx - k0);
#pragma unroll 4
      for (int s = 0; s < nb; ++s) {
        const long long c = __shfl_sync(kFull, ci, base + s);
        const T a = __shfl_sync(kFull, av, base + s);
        const T d = DERIV ? __shfl_sync(kFull, dv, base + s) : T(0);
        if (k0 + s < cnt) add(c, a, d);
      }
    }
  } else {
    for (int k0 = 0; k0 < mx; k0 += LPR * U) {
      int ci[U];
      T av[U], dv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int kk = k0 + u * LPR + g.l;
        ci[u] = 0;
        av[u] = T(0);
        dv[u] = T(0);
        if (kk < cnt) {
          ci[u] = __ldg(op.col + kb + kk);
          av[u] = __ldg(off + kb + kk);
          if (DERIV) dv[u] = __ldg(doff + kb + kk);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int s = 0; s < LPR; ++s) {
          const long long c = __shfl_sync(kFull, ci[u], base + s);
          const T a = __shfl_sync(kFull, av[u], base + s);
          const T d = DERIV ? __shfl_sync(kFull, dv[u], base + s) : T(0);
          if (k0 + u * LPR + s < cnt) add(c, a, d);
        }
    }
  }
}

// Grid used by every SLQ kernel (partial rows are indexed by blockIdx.x).
int slq_grid();

}  // namespace slq
}  // namespace lg
