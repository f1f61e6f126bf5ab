// lg_pool.h — the library's device memory pools (lg_pool.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

namespace lg {

// One stream-ordered memory pool per device that keeps its memory between
// calls (release threshold: never), so plans created and destroyed in a loop,
// and the adjoint's workspace, map no memory after the first call.
cudaError_t pool_for(int dev, cudaMemPool_t* out);

// `bytes` from the current device's pool, ordered on `st`; when the device
// is out of memory, the pools' unused memory goes back to the driver and the
// allocation is tried once more.
cudaError_t pool_alloc(void** p, size_t bytes, cudaStream_t st);

// Back to the pool, ordered on `st` (the memory is reused only after the work
// queued on `st` before this call).
void pool_free(void* p, cudaStream_t st);

}  // namespace lg
