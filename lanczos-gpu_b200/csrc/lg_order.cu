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

// ---------------------------------------------------------------------------
// Cuthill-McKee order (host).  Inside every BFS level the vertices follow the
// order of the vertices that discovered them (neighbours by increasing
// degree), so consecutive rows have neighbours that are themselves close
// together: a warp's gathers hit the same L1 lines and the rows of a CTA
// touch a narrow window of the block.  Each connected component starts from a
// pseudo-peripheral vertex (the last vertex reached by a BFS from its
// lowest-numbered vertex); components follow one another in order of that
// lowest vertex.
// ---------------------------------------------------------------------------
#include <algorithm>
#include <vector>

extern "C" int lg_graph_cm_order(int n, const int* rowptr, const int* col, int* perm) {
  if (n < 1 || !rowptr || !perm || (rowptr[n] > 0 && !col) || rowptr[0] != 0) {
    g_last_error = "lg_graph_cm_order: invalid arguments";
    return LG_ERR_INVALID;
  }
  for (int v = 0; v < n; ++v)
    if (rowptr[v + 1] < rowptr[v]) {
      g_last_error = "lg_graph_cm_order: row_ptr is not monotone";
      return LG_ERR_INVALID;
    }
  const long long nnz = rowptr[n];
  for (long long k = 0; k < nnz; ++k)
    if (col[k] < 0 || col[k] >= n) {
      g_last_error = "lg_graph_cm_order: column index out of range";
      return LG_ERR_INVALID;
    }
  std::vector<int> stamp((size_t)n, -1);   // BFS of the component search
  std::vector<char> placed((size_t)n, 0);
  std::vector<int> queue;
  queue.reserve((size_t)n);
  std::vector<int> nb;
  auto degree = [&](int v) { return rowptr[v + 1] - rowptr[v]; };
  int pos = 0, comp = 0;
  for (int root = 0; root < n; ++root) {
    if (placed[root]) continue;
    // pseudo-peripheral start: the last vertex a BFS from `root` reaches
    queue.clear();
    queue.push_back(root);
    stamp[root] = comp;
    for (size_t h = 0; h < queue.size(); ++h) {
      const int u = queue[h];
      for (int k = rowptr[u]; k < rowptr[u + 1]; ++k) {
        const int v = col[k];
        if (stamp[v] != comp && !placed[v]) {
          stamp[v] = comp;
          queue.push_back(v);
        }
      }
    }
    const int start = queue.back();
    ++comp;
    // Cuthill-McKee from `start`
    const int first = pos;
    perm[pos++] = start;
    placed[start] = 1;
    for (int h = first; h < pos; ++h) {
      const int u = perm[h];
      nb.clear();
      for (int k = rowptr[u]; k < rowptr[u + 1]; ++k) {
        const int v = col[k];
        if (!placed[v]) {
          placed[v] = 1;
          nb.push_back(v);
        }
      }
      std::sort(nb.begin(), nb.end(), [&](int a, int b) {
        const int da = degree(a), db = degree(b);
        return da != db ? da < db : a < b;
      });
      for (int v : nb) perm[pos++] = v;
    }
  }
  return pos == n ? LG_OK : LG_ERR_NUMERIC;
}
