// lg_staging.h — copies of pageable host memory through the pinned staging
// pool (lg_staging.cu).  Both return after the copy is complete.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

namespace lg {
cudaError_t staged_h2d(void* dst_dev, const void* src_host, size_t bytes, cudaStream_t st);
cudaError_t staged_d2h(void* dst_host, const void* src_dev, size_t bytes, cudaStream_t st);
}  // namespace lg
