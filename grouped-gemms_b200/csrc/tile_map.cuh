// Device-built routing tables with the layout of the reference's
// _build_expt_data (kernels/forward.py:340-365, kernel :296-338):
//   out[0, E)            tokens per group           (hist)
//   out[E, 2E)           start row of each group    (offs_raw)
//   out[2E]              sum of cdiv(hist, block_m) (offs_pad_sum)
//   out[2E+1, ...)       (block << 16) | group for each m-tile, -1 after the last
// The GEMM kernels build the same table in shared memory in their prologue;
// this stand-alone form exists for callers (and tests) that want the map.
#pragma once

#include <cstdint>

namespace mxgg {

__global__ void tile_map_kernel(const int32_t* __restrict__ offs, int E, int block_m, int grid_m_ub,
                                int32_t* __restrict__ out) {
  const long long n = 2LL * E + 1 + grid_m_ub;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    if (i < 2LL * E) {
      const int g = (int)(i < E ? i : i - E);
      const int prev = g > 0 ? offs[g - 1] : 0;
      out[i] = i < E ? offs[g] - prev : prev;
      continue;
    }
    int prev = 0, cum = 0, value = -1;
    const int pid = (int)(i - 2LL * E - 1);
    for (int e = 0; e < E; ++e) {
      const int off = offs[e];
      const int h = off - prev;
      const int blocks = (h + block_m - 1) / block_m;
      const int nxt = cum + blocks;
      if (pid >= 0 && pid >= cum && pid < nxt) value = ((pid - cum) << 16) | e;
      cum = nxt;
      prev = off;
    }
    out[i] = (i == 2LL * E) ? cum : value;
  }
}

}  // namespace mxgg
