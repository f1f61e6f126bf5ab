// lg_csr.cuh — CSR row kernels shared by the SpMV, CG and SLQ paths.
#pragma once

#include "lg_common.cuh"

namespace lg {

// Dot product of CSR row `row` with the gathered vector x, computed by a group
// of L lanes (L a power of two <= 32, groups aligned inside the warp); the
// result is valid in every lane of the group.  All 32 lanes must call it.
//
// Rows longer than kLongRow nonzeros are cut at kLongRow when `capped`; the
// rest of such a row is summed by long_rows_finish (lg_spmv.cu), so one
// power-law row cannot hold a whole product back.
constexpr int kLongRow = 2048;

template <typename VT, int L>
__device__ __forceinline__ double row_dot(const int* __restrict__ rowptr, const int* __restrict__ col,
                                          const VT* __restrict__ val, const double* __restrict__ x, int row,
                                          bool valid, int lane, bool capped = false) {
  double acc = 0.0;
  if (valid) {
    const int b = __ldg(rowptr + row);
    int e = __ldg(rowptr + row + 1);
    if (capped && e - b > kLongRow) e = b + kLongRow;
    for (int k = b + lane; k < e; k += L) acc += (double)__ldg(val + k) * __ldg(x + __ldg(col + k));
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace lg
