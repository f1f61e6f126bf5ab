// lg_knn.cu — exact k nearest neighbours of a point cloud and the kNN graph
// Laplacian L = D - A, built on the GPU.
//
// Replaces the graph construction of the reference's driver (src/main.cu:
// 30-124: brute-force O(n^2) distances on the host, partial_sort of
// (dist2, j) pairs per point, union symmetrisation, L = D - A with the
// diagonal at its sorted position) and of its large-graph generator
// (benchmark/generate_large_laplacian.py:30-66: scipy cKDTree query,
// exp(-d^2 / (4 bw^2)) weights, A.maximum(A.T), L = D - A).
//
// Neighbour order is ascending (squared distance, index): the order
// partial_sort gives the driver's pairs, so ties go to the smaller index and
// the result is a deterministic function of the points.  Distances are
// sums of squared coordinate differences in fp64, in coordinate order and
// without fused multiply-adds, so they equal a plain host loop bit for bit.
//
// Two searches:
//   * cells (dim <= 3): the points are binned into a uniform grid of about
//     max(2, k/2) points per cell (counting sort on the device); one thread
//     per point scans the cells in rings of growing Chebyshev radius and stops
//     when its k-th distance is below the distance to every unscanned cell.
//     O(n k) work for the uniform clouds of the reference's generators.
//   * brute (any dim <= 32): CTAs stream tiles of all points through shared
//     memory; each thread holds one query point in registers and keeps its k
//     best in a list that a candidate enters only when it beats the current
//     k-th entry.  O(n^2 dim) fp64 work, for the dim-10 clouds where a grid
//     does not prune.
// The Laplacian assembly counts, per row, the reverse edges that the row's
// own list lacks (j lists i, i does not list j), scans the row lengths, drops
// every entry in place and sorts each row by column; the degree is the
// sequential sum of the row's weights in column order (the order of a CSR
// row-sum), and off-diagonals are -w.
#include "../../include/lanczos_b200.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

namespace lg {
extern thread_local std::string g_last_error;

namespace {

constexpr int kKnnMaxK = 64;
constexpr int kKnnMaxDimBrute = 32;
constexpr int kBruteTileDoubles = 4096;   // 32 KB of points per shared-memory tile

// Ordered insertion of (s, j) into the k-best list (bd, bi) holding cnt
// entries; the list stays sorted by (distance, index).
template <int KMAX>
__device__ __forceinline__ void knn_insert(double (&bd)[KMAX], int (&bi)[KMAX], int& cnt, int k, double s, int j) {
  int p = cnt < k ? cnt++ : k - 1;
  while (p > 0 && (bd[p - 1] > s || (bd[p - 1] == s && bi[p - 1] > j))) {
    bd[p] = bd[p - 1];
    bi[p] = bi[p - 1];
    --p;
  }
  bd[p] = s;
  bi[p] = j;
}

__device__ __forceinline__ bool knn_better(double s, int j, double ws, int wj) {
  return s < ws || (s == ws && j < wj);
}

// The cell coordinate of x along one axis; the binning kernel and the search
// kernel both call this, so a point is searched from the cell it was stored in.
__device__ __forceinline__ int cell_coord(double x, double lo, double cell, int dim) {
  int c = (int)floor((x - lo) / cell);
  return min(max(c, 0), dim - 1);
}

template <int D>
__global__ void knn_bin_kernel(int n, const double* __restrict__ pts, int3 dims, double3 lo, double cell,
                               int* __restrict__ cell_id, int* __restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int dv[3] = {dims.x, dims.y, dims.z};
  const double lv[3] = {lo.x, lo.y, lo.z};
  int c[3] = {0, 0, 0};
#pragma unroll
  for (int d = 0; d < D; ++d) c[d] = cell_coord(pts[(size_t)i * D + d], lv[d], cell, dv[d]);
  const int id = (c[2] * dv[1] + c[1]) * dv[0] + c[0];
  cell_id[i] = id;
  atomicAdd(&counts[id], 1);
}

template <int D>
__global__ void knn_scatter_kernel(int n, const double* __restrict__ pts, const int* __restrict__ cell_id,
                                   const int* __restrict__ cell_start, int* __restrict__ cursor,
                                   double* __restrict__ pts_sorted, int* __restrict__ orig) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int id = cell_id[i];
  const int pos = cell_start[id] + atomicAdd(&cursor[id], 1);
#pragma unroll
  for (int d = 0; d < D; ++d) pts_sorted[(size_t)pos * D + d] = pts[(size_t)i * D + d];
  orig[pos] = i;
}

// Exclusive scan of counts[0..m) into out[0..m] (out[m] = total), one CTA of
// 1024 threads, each summing a contiguous chunk.  Used for cell starts and
// row pointers; m up to a few 10^7.
__global__ void __launch_bounds__(1024) scan_exclusive_kernel(int m, const int* __restrict__ counts,
                                                              int* __restrict__ out, long long* __restrict__ total) {
  __shared__ long long part[1024];
  const int t = threadIdx.x;
  const long long chunk = ((long long)m + 1023) / 1024;
  const long long b = t * chunk, e = b + chunk < m ? b + chunk : (long long)m;
  long long s = 0;
  for (long long i = b; i < e; ++i) s += counts[i];
  part[t] = s;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {   // Hillis-Steele inclusive scan of the chunk sums
    const long long v = t >= off ? part[t - off] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  long long run = part[t] - s;
  for (long long i = b; i < e; ++i) {
    out[i] = (int)run;
    run += counts[i];
  }
  if (t == 1023) {
    out[m] = (int)part[1023];
    if (total) *total = part[1023];
  }
}

template <int D, int KMAX>
__global__ void __launch_bounds__(128)
knn_cells_kernel(int n, int k, const double* __restrict__ pts, const int* __restrict__ orig,
                 const int* __restrict__ cell_start, int3 dims, double3 lo, double cell,
                 long long* __restrict__ out_idx, double* __restrict__ out_d2) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double bd[KMAX];
  int bi[KMAX];
  int cnt = 0;
  double x[3] = {0.0, 0.0, 0.0};
#pragma unroll
  for (int d = 0; d < D; ++d) x[d] = pts[(size_t)i * D + d];
  const int dv[3] = {dims.x, D > 1 ? dims.y : 1, D > 2 ? dims.z : 1};
  const double lv[3] = {lo.x, lo.y, lo.z};
  int c[3] = {0, 0, 0};
#pragma unroll
  for (int d = 0; d < D; ++d) c[d] = cell_coord(x[d], lv[d], cell, dv[d]);
  for (int r = 0;; ++r) {
    // every cell at Chebyshev distance exactly r from c, clipped to the grid
    const int z0 = D > 2 ? max(c[2] - r, 0) : 0, z1 = D > 2 ? min(c[2] + r, dv[2] - 1) : 0;
    const int y0 = D > 1 ? max(c[1] - r, 0) : 0, y1 = D > 1 ? min(c[1] + r, dv[1] - 1) : 0;
    const int x0 = max(c[0] - r, 0), x1 = min(c[0] + r, dv[0] - 1);
    for (int cz = z0; cz <= z1; ++cz)
      for (int cy = y0; cy <= y1; ++cy) {
        const bool inner = (D < 3 || abs(cz - c[2]) < r) && (D < 2 || abs(cy - c[1]) < r);
        for (int cx = x0; cx <= x1; ++cx) {
          if (inner && abs(cx - c[0]) < r) {   // interior of the ring: jump to its far side
            cx = c[0] + r - 1;
            continue;
          }
          const int id = (cz * dv[1] + cy) * dv[0] + cx;
          const int j1 = cell_start[id + 1];
          for (int j = cell_start[id]; j < j1; ++j) {
            if (j == i) continue;
            double s = 0.0;
#pragma unroll
            for (int d = 0; d < D; ++d) {
              const double t = pts[(size_t)j * D + d] - x[d];
              s = __dadd_rn(s, __dmul_rn(t, t));   // no contraction: the plain host sum, bit for bit
            }
            const int oj = orig[j];
            if (cnt == k && !knn_better(s, oj, bd[k - 1], bi[k - 1])) continue;
            knn_insert<KMAX>(bd, bi, cnt, k, s, oj);
          }
        }
      }
    // Distance from x to the nearest cell outside the scanned block, with a
    // margin for the rounding of the binning; infinite along clipped sides.
    double reach = INFINITY;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const double margin = 1e-9 * (fabs(x[d]) + fabs(lv[d]) + cell * (double)(abs(c[d]) + r + 1));
      if (c[d] - r > 0) reach = fmin(reach, x[d] - (lv[d] + (double)(c[d] - r) * cell) - margin);
      if (c[d] + r < dv[d] - 1) reach = fmin(reach, (lv[d] + (double)(c[d] + r + 1) * cell) - x[d] - margin);
    }
    if (reach == INFINITY) break;   // the block covers the grid: every point was seen
    if (cnt == k && reach > 0.0 && bd[k - 1] < reach * reach) break;
  }
  const int me = orig[i];
  for (int q = 0; q < k; ++q) {
    out_idx[(size_t)me * k + q] = q < cnt ? bi[q] : -1;
    out_d2[(size_t)me * k + q] = q < cnt ? bd[q] : 0.0;
  }
}

template <int DMAX, int KMAX>
__global__ void __launch_bounds__(128)
knn_brute_kernel(int n, int dim, int k, const double* __restrict__ pts, long long* __restrict__ out_idx,
                 double* __restrict__ out_d2) {
  extern __shared__ double tile[];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = i < n;
  double x[DMAX];
#pragma unroll
  for (int d = 0; d < DMAX; ++d) x[d] = (active && d < dim) ? pts[(size_t)i * dim + d] : 0.0;
  double bd[KMAX];
  int bi[KMAX];
  int cnt = 0;
  double worst = INFINITY;
  int worst_i = 0x7fffffff;
  const int tp = kBruteTileDoubles / dim;   // points per tile
  for (int base = 0; base < n; base += tp) {
    const int cntp = min(tp, n - base);
    __syncthreads();
    const size_t off = (size_t)base * dim;
    for (int t = threadIdx.x; t < cntp * dim; t += blockDim.x) tile[t] = pts[off + t];
    __syncthreads();
    if (!active) continue;
    for (int p = 0; p < cntp; ++p) {
      const double* q = tile + p * dim;
      double s = 0.0;
#pragma unroll
      for (int d = 0; d < DMAX; ++d)
        if (d < dim) {
          const double t = q[d] - x[d];
          s = __dadd_rn(s, __dmul_rn(t, t));
        }
      const int j = base + p;
      if (j == i) continue;
      if (cnt == k && !knn_better(s, j, worst, worst_i)) continue;
      knn_insert<KMAX>(bd, bi, cnt, k, s, j);
      if (cnt == k) {
        worst = bd[k - 1];
        worst_i = bi[k - 1];
      }
    }
  }
  if (!active) return;
  for (int q = 0; q < k; ++q) {
    out_idx[(size_t)i * k + q] = q < cnt ? bi[q] : -1;
    out_d2[(size_t)i * k + q] = q < cnt ? bd[q] : 0.0;
  }
}

// Per-block minimum and maximum of every coordinate: part[b * 2 dim + d] and
// part[b * 2 dim + dim + d]; *bad = 1 on a NaN or infinite coordinate.
__global__ void knn_bounds_kernel(int n, int dim, const double* __restrict__ pts, double* __restrict__ part,
                                  int* __restrict__ bad) {
  __shared__ double smin[256], smax[256];
  for (int d = 0; d < dim; ++d) {
    double mn = INFINITY, mx = -INFINITY;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
      const double v = pts[(size_t)i * dim + d];
      if (!isfinite(v)) *bad = 1;
      mn = fmin(mn, v);
      mx = fmax(mx, v);
    }
    smin[threadIdx.x] = mn;
    smax[threadIdx.x] = mx;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
      if ((int)threadIdx.x < s) {
        smin[threadIdx.x] = fmin(smin[threadIdx.x], smin[threadIdx.x + s]);
        smax[threadIdx.x] = fmax(smax[threadIdx.x], smax[threadIdx.x + s]);
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      part[(size_t)blockIdx.x * 2 * dim + d] = smin[0];
      part[(size_t)blockIdx.x * 2 * dim + dim + d] = smax[0];
    }
    __syncthreads();
  }
}

// ---- Laplacian assembly ------------------------------------------------------

// Checks every directed edge (i -> j = idx[i k + q]) and counts, for row j,
// the edges whose reverse j lists no (i not in j's list).  *bad = 1 on an
// index outside [0, n), a self edge or a neighbour listed twice.
__global__ void lap_count_kernel(int n, int k, const long long* __restrict__ idx, int* __restrict__ extra,
                                 int* __restrict__ bad) {
  const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= (long long)n * k) return;
  const int i = (int)(e / k), q = (int)(e % k);
  const long long jl = idx[e];
  if (jl < 0 || jl >= n || jl == i) {
    *bad = 1;
    return;
  }
  for (int p = 0; p < q; ++p)
    if (idx[(size_t)i * k + p] == jl) {
      *bad = 1;
      return;
    }
  const int j = (int)jl;
  bool found = false;
  for (int p = 0; p < k && !found; ++p) found = idx[(size_t)j * k + p] == i;
  if (!found) atomicAdd(&extra[j], 1);
}

__global__ void lap_lengths_kernel(int n, int k, int* __restrict__ len) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) len[i] += k + 1;   // own neighbours + diagonal + reverse-only edges
}

// Row i holds its own k neighbours at rowptr[i] .. +k, the diagonal at +k and
// the reverse-only edges after it (in atomic order; the row sort fixes it).
__global__ void lap_fill_kernel(int n, int k, const long long* __restrict__ idx, const double* __restrict__ d2,
                                double denom, const int* __restrict__ rowptr, int* __restrict__ cursor,
                                int* __restrict__ col, double* __restrict__ val) {
  const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= (long long)n * k) return;
  const int i = (int)(e / k), q = (int)(e % k);
  const long long jl = idx[e];
  if (jl < 0 || jl >= n) return;   // lists are checked by lg_knn_laplacian_rows; never write outside
  const int j = (int)jl;
  const double w = exp(-d2[e] / denom);
  col[rowptr[i] + q] = j;
  val[rowptr[i] + q] = -w;
  if (q == 0) {
    col[rowptr[i] + k] = i;
    val[rowptr[i] + k] = 0.0;
  }
  bool found = false;
  for (int p = 0; p < k && !found; ++p) found = idx[(size_t)j * k + p] == i;
  if (!found) {
    const int slot = rowptr[j] + k + 1 + atomicAdd(&cursor[j], 1);
    if (slot < rowptr[j + 1]) {
      col[slot] = i;
      val[slot] = -w;
    }
  }
}

// Sorts row i by column (insertion sort: kNN rows are short) and sets the
// diagonal to the sequential sum of the row's weights in column order.
__global__ void lap_sort_rows_kernel(int n, const int* __restrict__ rowptr, int* __restrict__ col,
                                     double* __restrict__ val) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int b = rowptr[i], e = rowptr[i + 1];
  for (int p = b + 1; p < e; ++p) {
    const int c = col[p];
    const double v = val[p];
    int q = p;
    while (q > b && col[q - 1] > c) {
      col[q] = col[q - 1];
      val[q] = val[q - 1];
      --q;
    }
    col[q] = c;
    val[q] = v;
  }
  double deg = 0.0;
  int dpos = b;
  for (int p = b; p < e; ++p) {
    if (col[p] == i)
      dpos = p;
    else
      deg += -val[p];
  }
  val[dpos] = deg;
}

int pick_kmax(int k) { return k <= 16 ? 16 : (k <= 32 ? 32 : 64); }

// Device scratch from the stream-ordered allocator, released on scope exit.
struct Scratch {
  cudaStream_t st;
  std::vector<void*> ptrs;
  explicit Scratch(cudaStream_t s) : st(s) {}
  template <class T>
  cudaError_t get(T** p, size_t count) {
    void* q = nullptr;
    const cudaError_t e = cudaMallocAsync(&q, std::max<size_t>(count, 1) * sizeof(T), st);
    if (e == cudaSuccess) ptrs.push_back(q);
    *p = static_cast<T*>(q);
    return e;
  }
  ~Scratch() {
    for (void* q : ptrs) cudaFreeAsync(q, st);
  }
};

#define KNN_TRY(expr)                                                     \
  do {                                                                    \
    const cudaError_t e_ = (expr);                                        \
    if (e_ != cudaSuccess) {                                              \
      g_last_error = std::string(fname) + ": " + cudaGetErrorString(e_);  \
      return LG_ERR_CUDA;                                                 \
    }                                                                     \
  } while (0)

template <int D>
int knn_cells(int n, int k, const double* pts, const double* lo_h, const double* ext_h, long long* out_idx,
              double* out_d2, cudaStream_t st) {
  static const char* fname = "lg_knn";
  // cells of about max(2, k/2) points over the axes with a positive extent
  const double per_cell = std::max(2.0, k / 2.0);
  double vol = 1.0;
  int live = 0;
  for (int d = 0; d < D; ++d)
    if (ext_h[d] > 0.0) {
      vol *= ext_h[d];
      ++live;
    }
  double cell = live ? std::pow(vol * per_cell / n, 1.0 / live) : 1.0;
  if (!(cell > 0.0) || !std::isfinite(cell)) cell = std::max({ext_h[0], D > 1 ? ext_h[1] : 0.0, D > 2 ? ext_h[2] : 0.0, 1.0});
  int dims[3] = {1, 1, 1};
  for (int grow = 0;; ++grow) {
    long long total = 1;
    for (int d = 0; d < D; ++d) {
      const double c = ext_h[d] > 0.0 ? std::ceil(ext_h[d] / cell) : 1.0;
      dims[d] = (int)std::min(std::max(c, 1.0), 1048576.0);
      total *= dims[d];
    }
    if (total <= 2LL * n + 64 || grow > 60) break;
    cell *= 1.25;   // an elongated cloud: coarser cells until the grid fits
  }
  if ((long long)dims[0] * dims[1] * dims[2] > 0x7ffffffeLL) {
    g_last_error = "lg_knn: the point cloud is too spread out for a cell grid (use the brute-force search)";
    return LG_ERR_INVALID;
  }
  const int ncells = dims[0] * dims[1] * dims[2];
  const int3 gd = make_int3(dims[0], dims[1], dims[2]);
  const double3 glo = make_double3(lo_h[0], D > 1 ? lo_h[1] : 0.0, D > 2 ? lo_h[2] : 0.0);
  Scratch sc(st);
  int *cell_id, *counts, *cell_start, *cursor, *orig;
  double* sorted;
  KNN_TRY(sc.get(&cell_id, n));
  KNN_TRY(sc.get(&counts, ncells));
  KNN_TRY(sc.get(&cell_start, (size_t)ncells + 1));
  KNN_TRY(sc.get(&cursor, ncells));
  KNN_TRY(sc.get(&orig, n));
  KNN_TRY(sc.get(&sorted, (size_t)n * D));
  KNN_TRY(cudaMemsetAsync(counts, 0, sizeof(int) * ncells, st));
  KNN_TRY(cudaMemsetAsync(cursor, 0, sizeof(int) * ncells, st));
  const int g = (n + 255) / 256;
  knn_bin_kernel<D><<<g, 256, 0, st>>>(n, pts, gd, glo, cell, cell_id, counts);
  scan_exclusive_kernel<<<1, 1024, 0, st>>>(ncells, counts, cell_start, nullptr);
  knn_scatter_kernel<D><<<g, 256, 0, st>>>(n, pts, cell_id, cell_start, cursor, sorted, orig);
  const int gs = (n + 127) / 128;
  switch (pick_kmax(k)) {
    case 16:
      knn_cells_kernel<D, 16><<<gs, 128, 0, st>>>(n, k, sorted, orig, cell_start, gd, glo, cell, out_idx, out_d2);
      break;
    case 32:
      knn_cells_kernel<D, 32><<<gs, 128, 0, st>>>(n, k, sorted, orig, cell_start, gd, glo, cell, out_idx, out_d2);
      break;
    default:
      knn_cells_kernel<D, 64><<<gs, 128, 0, st>>>(n, k, sorted, orig, cell_start, gd, glo, cell, out_idx, out_d2);
      break;
  }
  KNN_TRY(cudaGetLastError());
  return LG_OK;
}

template <int DMAX>
void knn_brute_launch(int n, int dim, int k, const double* pts, long long* out_idx, double* out_d2,
                      cudaStream_t st) {
  const int g = (n + 127) / 128;
  const size_t smem = sizeof(double) * kBruteTileDoubles;
  switch (pick_kmax(k)) {
    case 16: knn_brute_kernel<DMAX, 16><<<g, 128, smem, st>>>(n, dim, k, pts, out_idx, out_d2); break;
    case 32: knn_brute_kernel<DMAX, 32><<<g, 128, smem, st>>>(n, dim, k, pts, out_idx, out_d2); break;
    default: knn_brute_kernel<DMAX, 64><<<g, 128, smem, st>>>(n, dim, k, pts, out_idx, out_d2); break;
  }
}

}  // namespace
}  // namespace lg

using namespace lg;

extern "C" int lg_knn(int n, int dim, int k, const double* pts, long long* out_idx, double* out_d2, int method,
                      void* stream) {
  static const char* fname = "lg_knn";
  if (n < 2 || dim < 1 || k < 1 || k > kKnnMaxK || k >= n || !pts || !out_idx || !out_d2 || method < 0 ||
      method > 2) {
    g_last_error = "lg_knn: invalid arguments (n >= 2, dim >= 1, 1 <= k <= min(64, n - 1), method 0/1/2)";
    return LG_ERR_INVALID;
  }
  if (method == LG_KNN_CELLS && dim > 3) {
    g_last_error = "lg_knn: the cell search takes dim <= 3";
    return LG_ERR_INVALID;
  }
  const bool cells = method == LG_KNN_CELLS || (method == LG_KNN_AUTO && dim <= 3);
  if (!cells && dim > kKnnMaxDimBrute) {
    g_last_error = "lg_knn: the brute-force search takes dim <= 32";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // bounds and finiteness of the coordinates
  const int nb = std::min(256, (n + 255) / 256);
  std::vector<double> part((size_t)nb * 2 * dim);
  int bad_h = 0;
  {
    Scratch sc(st);
    double* d_part;
    int* d_bad;
    KNN_TRY(sc.get(&d_part, part.size()));
    KNN_TRY(sc.get(&d_bad, 1));
    KNN_TRY(cudaMemsetAsync(d_bad, 0, sizeof(int), st));
    knn_bounds_kernel<<<nb, 256, 0, st>>>(n, dim, pts, d_part, d_bad);
    KNN_TRY(cudaGetLastError());
    KNN_TRY(cudaMemcpyAsync(part.data(), d_part, sizeof(double) * part.size(), cudaMemcpyDeviceToHost, st));
    KNN_TRY(cudaMemcpyAsync(&bad_h, d_bad, sizeof(int), cudaMemcpyDeviceToHost, st));
    KNN_TRY(cudaStreamSynchronize(st));
  }
  if (bad_h) {
    g_last_error = "lg_knn: the points must be finite";
    return LG_ERR_INVALID;
  }
  if (!cells) {
    if (dim <= 4) knn_brute_launch<4>(n, dim, k, pts, out_idx, out_d2, st);
    else if (dim <= 8) knn_brute_launch<8>(n, dim, k, pts, out_idx, out_d2, st);
    else if (dim <= 16) knn_brute_launch<16>(n, dim, k, pts, out_idx, out_d2, st);
    else knn_brute_launch<32>(n, dim, k, pts, out_idx, out_d2, st);
    KNN_TRY(cudaGetLastError());
    return LG_OK;
  }
  double lo[3] = {0, 0, 0}, ext[3] = {0, 0, 0};
  for (int d = 0; d < dim; ++d) {
    double mn = INFINITY, mx = -INFINITY;
    for (int b = 0; b < nb; ++b) {
      mn = std::min(mn, part[(size_t)b * 2 * dim + d]);
      mx = std::max(mx, part[(size_t)b * 2 * dim + dim + d]);
    }
    lo[d] = mn;
    ext[d] = mx - mn;
  }
  switch (dim) {
    case 1: return knn_cells<1>(n, k, pts, lo, ext, out_idx, out_d2, st);
    case 2: return knn_cells<2>(n, k, pts, lo, ext, out_idx, out_d2, st);
    default: return knn_cells<3>(n, k, pts, lo, ext, out_idx, out_d2, st);
  }
}

extern "C" int lg_knn_laplacian_rows(int n, int k, const long long* idx, int* rowptr, long long* nnz, void* stream) {
  static const char* fname = "lg_knn_laplacian_rows";
  if (n < 2 || k < 1 || k >= n || !idx || !rowptr || !nnz) {
    g_last_error = "lg_knn_laplacian_rows: invalid arguments";
    return LG_ERR_INVALID;
  }
  if ((long long)n * k > 0x7fffffffLL) {
    g_last_error = "lg_knn_laplacian_rows: n * k must fit in int32";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Scratch sc(st);
  int *len, *bad;
  long long* total;
  KNN_TRY(sc.get(&len, n));
  KNN_TRY(sc.get(&bad, 1));
  KNN_TRY(sc.get(&total, 1));
  KNN_TRY(cudaMemsetAsync(len, 0, sizeof(int) * n, st));
  KNN_TRY(cudaMemsetAsync(bad, 0, sizeof(int), st));
  const long long edges = (long long)n * k;
  lap_count_kernel<<<(unsigned)((edges + 255) / 256), 256, 0, st>>>(n, k, idx, len, bad);
  lap_lengths_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, k, len);
  scan_exclusive_kernel<<<1, 1024, 0, st>>>(n, len, rowptr, total);
  KNN_TRY(cudaGetLastError());
  int bad_h = 0;
  long long tot_h = 0;
  KNN_TRY(cudaMemcpyAsync(&bad_h, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
  KNN_TRY(cudaMemcpyAsync(&tot_h, total, sizeof(long long), cudaMemcpyDeviceToHost, st));
  KNN_TRY(cudaStreamSynchronize(st));
  if (bad_h) {
    g_last_error = "lg_knn_laplacian_rows: neighbour lists must hold distinct indices in [0, n) other than the row";
    return LG_ERR_INVALID;
  }
  if (tot_h > 0x7fffffffLL) {
    g_last_error = "lg_knn_laplacian_rows: nnz must fit in int32";
    return LG_ERR_INVALID;
  }
  *nnz = tot_h;
  return LG_OK;
}

extern "C" int lg_knn_laplacian_fill(int n, int k, const long long* idx, const double* d2, double denom,
                                     const int* rowptr, int* col, double* val, void* stream) {
  static const char* fname = "lg_knn_laplacian_fill";
  if (n < 2 || k < 1 || k >= n || !idx || !d2 || !(denom > 0.0) || !rowptr || !col || !val) {
    g_last_error = "lg_knn_laplacian_fill: invalid arguments (denom > 0)";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Scratch sc(st);
  int* cursor;
  KNN_TRY(sc.get(&cursor, n));
  KNN_TRY(cudaMemsetAsync(cursor, 0, sizeof(int) * n, st));
  const long long edges = (long long)n * k;
  lap_fill_kernel<<<(unsigned)((edges + 255) / 256), 256, 0, st>>>(n, k, idx, d2, denom, rowptr, cursor, col, val);
  lap_sort_rows_kernel<<<(n + 127) / 128, 128, 0, st>>>(n, rowptr, col, val);
  KNN_TRY(cudaGetLastError());
  return LG_OK;
}
