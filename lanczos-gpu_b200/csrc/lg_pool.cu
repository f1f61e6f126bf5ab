// lg_pool.cu — device memory pools of the library (see lg_pool.h).
#include "lg_pool.h"

#include <mutex>

namespace lg {

namespace {
constexpr int kMaxPoolDevices = 64;
cudaMemPool_t g_pools[kMaxPoolDevices] = {};
std::mutex g_pool_mu;
}  // namespace

cudaError_t pool_for(int dev, cudaMemPool_t* out) {
  if (dev < 0 || dev >= kMaxPoolDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_pool_mu);
  if (!g_pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    cudaError_t e = cudaMemPoolCreate(&p, &props);
    if (e != cudaSuccess) return e;
    unsigned long long keep = ~0ull;
    e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) {
      cudaMemPoolDestroy(p);
      return e;
    }
    g_pools[dev] = p;
  }
  *out = g_pools[dev];
  return cudaSuccess;
}

cudaError_t pool_alloc(void** p, size_t bytes, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaMemPool_t pool = nullptr;
  if ((e = pool_for(dev, &pool)) != cudaSuccess) return e;
  e = cudaMallocFromPoolAsync(p, bytes, pool, st);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    // memory the pool keeps but nobody uses goes back to the driver
    cudaStreamSynchronize(st);
    cudaMemPoolTrimTo(pool, 0);
    e = cudaMallocFromPoolAsync(p, bytes, pool, st);
  }
  return e;
}

void pool_free(void* p, cudaStream_t st) {
  if (p) cudaFreeAsync(p, st);
}

}  // namespace lg
