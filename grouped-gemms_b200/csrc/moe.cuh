// MoE combine: out[t] = sum_j weights[t, j] * y[pos[t, j]] for the top-k rows
// each token was routed to (fp32 sum in choice order, bf16 out).  One warp per
// token, 16-byte loads and stores; HBM-bound (k reads + 1 write per element).
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace mxgg {

__global__ void __launch_bounds__(256) combine_topk_bf16(const __nv_bfloat16* __restrict__ y,
                                                         const int64_t* __restrict__ pos,
                                                         const float* __restrict__ weights, long long y_rows,
                                                         int T, int N, int k, __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nwarps) {
    for (int c0 = lane * 8; c0 < N; c0 += 32 * 8) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
      for (int j = 0; j < k; ++j) {
        const long long r = __ldg(pos + t * k + j);
        const float w = __ldg(weights + t * k + j);
        if (r < 0 || r >= y_rows) continue;          // out-of-range positions contribute nothing
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(y + r * N + c0));
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] += w * __uint_as_float(wv[i] << 16);
          acc[2 * i + 1] += w * __uint_as_float(wv[i] & 0xFFFF0000u);
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(out + t * N + c0) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace mxgg
