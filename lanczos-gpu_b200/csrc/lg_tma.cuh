// lg_tma.cuh — a ring of shared-memory stages filled by TMA bulk copies.
//
// A stage holds one row tile of the column-major basis V: `ncols` column
// segments of T doubles each (plus, optionally, one extra vector segment).
// Warp 0 issues the copies (one cp.async.bulk per segment, completion counted
// on the stage's mbarrier); every thread waits on the barrier before reading.
// The waits are bounded (lg_common.cuh: mbar_wait_bounded): on a timeout the
// kernel records STATUS_TIMEOUT, lets in-flight copies land (bounded again)
// and returns, so no launch can hang the GPU.
#pragma once

#include "lg_common.cuh"

namespace lg {

struct TileRing {
  uint64_t* bar;     // S mbarriers
  double* buf;       // S stages of nseg * T doubles
  int S, T, ncols, ld;
  const double* V;
  const double* vec; // optional extra segment (may be null)

  __device__ int nseg() const { return ncols + (vec ? 1 : 0); }
  __device__ double* stage_ptr(int s) const { return buf + (size_t)s * nseg() * T; }

  __device__ void init_barriers() const {
    if (threadIdx.x == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
      mbar_init_fence();
    }
    __syncthreads();
  }

  // Called by all lanes of warp 0.
  __device__ void issue(int tile, int s) const {
    const int lane = threadIdx.x & 31;
    const size_t row0 = (size_t)tile * T;
    double* dst = stage_ptr(s);
    const uint32_t seg = (uint32_t)T * 8u;
    const int ns = nseg();
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bar[s], seg * (uint32_t)ns);
    }
    __syncwarp();
    for (int c = lane; c < ns; c += 32) {
      const double* src = (c < ncols) ? (V + (size_t)c * ld + row0) : (vec + row0);
      tma_load_1d(dst + (size_t)c * T, src, seg, &bar[s]);
    }
  }

  // Thread 0 waits (bounded) and publishes the outcome; then every thread
  // observes the completed phase.  Returns false on timeout (block-uniform).
  __device__ bool wait(int s, uint32_t parity, int* flag_smem, int* state, int site) const {
    if (threadIdx.x == 0) *flag_smem = mbar_wait_bounded(&bar[s], parity) ? 1 : 0;
    __syncthreads();
    const int ok = *flag_smem;
    if (ok) {
      mbar_wait_bounded(&bar[s], parity);  // already complete: returns at once
    } else if (threadIdx.x == 0) {
      atomicExch(&state[ST_ERRINFO], site);
      atomicExch(&state[ST_STATUS], STATUS_TIMEOUT);
    }
    return ok != 0;
  }

  // After a timeout: give copies still in flight a short, bounded chance to
  // land before the CTA exits.
  __device__ void drain(int it, int nt) const {
    if (threadIdx.x == 0) {
      for (int k = it; k < nt && k < it + S; ++k)
        mbar_wait_bounded(&bar[k % S], (uint32_t)((k / S) & 1), 20000000ll);
    }
    __syncthreads();
  }
};

}  // namespace lg
