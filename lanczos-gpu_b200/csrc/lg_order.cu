// lg_order.cu — breadth-first levels of a graph, for a locality ordering of
// the rows of a sparse operator.
//
// The SLQ sparse products gather, for every row, the probe rows of its
// neighbours (256 bytes each at 64 fp32 probes).  In the original order of a
// kNN graph those rows are scattered over the whole n x B block, which does
// not fit in L2, so every gather is a DRAM access.  Ordering the rows by BFS
// level from a peripheral vertex (the level structure behind Cuthill-McKee)
// puts every neighbour within the previous, the same or the next level, so
// the rows a CTA gathers were just touched by its neighbours in the grid and
// stay in L2.  Log-determinants and gradients do not depend on the order.
//
// Queue-based level-synchronous BFS: one launch per level reads the current
// frontier and claims unvisited neighbours with atomicCAS, appending them to
// the next frontier.  Levels run in batches between host checks of the
// frontier size; the host loop is bounded by n levels.  The frontier order
// inside a level is not deterministic, the level of every vertex is.
#include "lg_common.cuh"

#include "../../include/lanczos_b200.h"

#include <string>

namespace lg {
extern thread_local std::string g_last_error;

namespace {

__global__ void bfs_init_kernel(int n, int start, int* level, int* frontier, int* counts) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    level[i] = (i == start) ? 0 : -1;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    frontier[0] = start;
    counts[0] = 1;
    counts[1] = 0;
  }
}

// Expand the frontier of level `cur` (count in counts[cur & 1]) into the next
// one (counts[(cur + 1) & 1], zeroed by the previous level's kernel).
__global__ void bfs_level_kernel(const int* __restrict__ rowptr, const int* __restrict__ col, int* level,
                                 const int* __restrict__ frontier, int* __restrict__ next, int* counts, int cur) {
  const int fc = counts[cur & 1];
  int* ncount = counts + ((cur + 1) & 1);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < fc; i += (long long)gridDim.x * blockDim.x) {
    const int u = frontier[i];
    for (int k = rowptr[u]; k < rowptr[u + 1]; ++k) {
      const int v = col[k];
      if (atomicCAS(level + v, -1, cur + 1) == -1) next[atomicAdd(ncount, 1)] = v;
    }
  }
}

__global__ void bfs_reset_count_kernel(int* counts, int idx) { counts[idx] = 0; }

}  // namespace
}  // namespace lg

using namespace lg;

extern "C" int lg_graph_bfs_levels(int n, const int* rowptr, const int* col, int start, int* level, int* work,
                                   int* nlevels, void* stream) {
  if (n < 1 || !rowptr || !level || !work || !nlevels || start < 0 || start >= n) {
    g_last_error = "lg_graph_bfs_levels: invalid arguments";
    return LG_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* fr[2] = {work, work + n};
  int* counts = work + 2 * (size_t)n;       // two ints
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = 4 * (sms > 0 ? sms : 1), threads = 256;
  bfs_init_kernel<<<grid, threads, 0, st>>>(n, start, level, fr[0], counts);
  int cur = 0;
  int host_counts[2] = {1, 0};
  constexpr int kBatch = 16;
  while (cur < n) {
    for (int b = 0; b < kBatch; ++b, ++cur) {
      // next count slot is zero: set before this level by the reset below
      bfs_level_kernel<<<grid, threads, 0, st>>>(rowptr, col, level, fr[cur & 1], fr[(cur + 1) & 1], counts, cur);
      bfs_reset_count_kernel<<<1, 1, 0, st>>>(counts, cur & 1);
    }
    cudaError_t e = cudaMemcpyAsync(host_counts, counts, sizeof(host_counts), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      g_last_error = std::string("lg_graph_bfs_levels: ") + cudaGetErrorString(e);
      return LG_ERR_CUDA;
    }
    if (host_counts[cur & 1] == 0) break;
  }
  // the last level with a vertex: scan on the host would need the array; the
  // caller derives it from `level`.  Report the number of expansion rounds.
  *nlevels = cur;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_error = std::string("lg_graph_bfs_levels: ") + cudaGetErrorString(e);
    return LG_ERR_CUDA;
  }
  return LG_OK;
}
