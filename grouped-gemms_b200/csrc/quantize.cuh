// MX quantiser (FLOOR scaling, 32-element blocks) for sm_100a.
//
// Bit-exact restatement of the reference's utils.to_mx (utils.py:67-105):
//   amax    = max |x| over the block (NaN propagates, utils.py:86)
//   e       = biased exponent of max(amax, FLT_MIN)            (utils.py:88-92)
//   s       = clamp(e - emax, 0, 254)   emax = 8 (e4m3), 2 (e2m1)  (utils.py:93-95)
//   q       = cast(clamp(x * 2^(127 - s), -max, max))           (utils.py:97-101)
// x * 2^(127-s) equals the reference's x / 2^(s-127) exactly: both are the
// correctly rounded value of the same real number, and 2^(127-s) is a normal
// float for every reachable s.  NaN keeps its sign (0x7F / 0xFF), like the
// reference's CPU cast.
//
// Layout: each thread owns 8 consecutive elements (one 16-byte bf16 vector),
// four neighbouring lanes form a 32-block and reduce the amax with two xor
// shuffles; stores are 8-byte vectors.  The kernel is HBM-bound: it reads
// 2 B/elem (bf16), writes 1 B/elem + 1 B/32 elem.
//
// Two modes:
//   rows  : quantise along the contiguous last dim (the reference's to_mx).
//   cols  : quantise along the leading dim and write the transposed result
//           (to_mx(x.t().contiguous()) fused into one pass) -- the operand
//           layout the wgrad pass consumes (scales along tokens).
// Scales are written row-major (the reference layout) or, on request, in the
// 128x4 blocked scale-factor atom layout used by Blackwell block-scaled MMAs:
// over the whole matrix (kScaleBlocked), or per row segment (kScaleBlockedSeg:
// every segment starts a new 128-row slab -- the layout the grouped GEMM
// reads for forward A (segments = groups) and B (segments = experts)).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace mxgg {

enum : int { kInBF16 = 0, kInF16 = 1, kInF32 = 2 };
enum : int { kScaleRowMajor = 0, kScaleBlocked = 1, kScaleBlockedSeg = 2 };
constexpr int kMaxScaleSegments = 256;

// Row segments of a kScaleBlockedSeg scale tensor: device cumulative ends
// (offs, n segments) or, with offs null, uniform segments of seg_rows rows.
struct ScaleSegs {
  const int32_t* offs;
  int n;
  long long seg_rows;
};

// Per-CTA table of a ScaleSegs with device offsets: clamped, monotone
// segment starts, the end of the last segment and the exclusive prefix of the
// segments' 128-row slabs.
struct SegTable {
  int start[kMaxScaleSegments];
  int cum[kMaxScaleSegments + 1];
  int end;
};

__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

// 8 consecutive inputs -> float
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// scale byte from the (NaN-propagating) max of |x| bit patterns
__device__ __forceinline__ uint32_t floor_scale(uint32_t amax_bits, int emax) {
  const uint32_t b = max(amax_bits, 0x00800000u);     // clamp(min = FLT_MIN)
  const int e = (int)(b >> 23);                       // biased exponent (sign already clear)
  return (uint32_t)min(max(e - emax, 0), 254);
}

// e4m3 byte of x * mult, with the reference's clamp and NaN sign rule
__device__ __forceinline__ uint32_t e4m3_byte(float x, float mult) {
  if (x != x) return (__float_as_uint(x) >> 31) ? 0xFFu : 0x7Fu;
  float v = x * mult;
  v = fminf(fmaxf(v, -448.0f), 448.0f);
  return (uint32_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// Eight inputs of one 32-block -> eight e4m3 bytes (two words).  Blocks
// without NaN (amax bit pattern <= +inf) take the paired conversion: the
// satfinite cvt saturates exactly like the reference's clamp to +-448 followed
// by the cast (an infinite input lands on 448 too).  A block holding a NaN
// converts element by element so each NaN keeps its sign.
__device__ __forceinline__ uint2 e4m3x8(const float (&f)[8], float mult, uint32_t amax_bits) {
  if (amax_bits <= 0x7F800000u) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(f[2 * k] * mult, f[2 * k + 1] * mult), __NV_SATFINITE,
                                                __NV_E4M3);
    return make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
  }
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) lo |= e4m3_byte(f[k], mult) << (8 * k);
#pragma unroll
  for (int k = 0; k < 4; ++k) hi |= e4m3_byte(f[4 + k], mult) << (8 * k);
  return make_uint2(lo, hi);
}

// Eight inputs of one 32-block -> eight e2m1 nibbles (one word, element 2k in
// the low nibble of byte k, the layout the tensor cores and TMA's 4-bit types
// read).  MXFP4 has no counterpart in the reference: FLOOR scaling is extended
// with emax = 2, values saturate to +-6 and NaN becomes +6 (the hardware
// conversion's rule; e2m1 has no NaN).
__device__ __forceinline__ uint32_t e2m1x8(const float (&f)[8], float mult) {
  uint32_t w = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    w |= (uint32_t)__nv_cvt_float2_to_fp4x2(make_float2(f[2 * k] * mult, f[2 * k + 1] * mult), __NV_E2M1,
                                            cudaRoundNearest)
         << (8 * k);
  return w;
}

// offset of scale (r, c) of a (R, C) scale matrix in the blocked atom layout
__device__ __forceinline__ long long blocked_sf_offset(long long r, long long c, long long C) {
  const long long cb = (C + 3) / 4;
  const long long atom = (r / 128) * cb + (c / 4);
  return atom * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4);
}

// one warp fills `t` from segs.offs (rows: the scale matrix height)
__device__ __forceinline__ void build_seg_table(SegTable& t, const ScaleSegs& segs, long long rows) {
  const int lane = threadIdx.x & 31;
  int carry_max = 0, carry_sum = 0;
  for (int base = 0; base < segs.n; base += 32) {
    const int i = base + lane;
    int c = 0;
    if (i < segs.n) c = (int)min(max((long long)__ldg(segs.offs + i), 0LL), rows);
    int v = (i < segs.n) ? max(c, carry_max) : carry_max;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v = max(v, u);
    }
    int prev = __shfl_up_sync(0xffffffffu, v, 1);
    if (lane == 0) prev = carry_max;
    const int n128 = (i < segs.n) ? (v - prev + 127) / 128 : 0;
    int incl = n128;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (i < segs.n) {
      t.start[i] = prev;
      t.cum[i] = carry_sum + incl - n128;
    }
    carry_max = __shfl_sync(0xffffffffu, v, 31);
    carry_sum += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    t.cum[segs.n] = carry_sum;
    t.end = carry_max;
  }
}

// Offset of scale (r, c) of a (R, C) scale matrix in the per-segment blocked
// layout, or -1 for a row no segment holds (at or past the last segment's
// end).  Segment g's rows fill slabs cum[g], cum[g] + 1, ...: row r of the
// segment is row r % 128 of slab cum[g] + r / 128.
__device__ __forceinline__ long long blocked_seg_sf_offset(long long r, long long c, long long C, const ScaleSegs& segs,
                                                           const SegTable& t) {
  long long slab, rr;
  if (!segs.offs) {
    const long long g = r / segs.seg_rows;
    if (g >= segs.n) return -1;
    rr = r - g * segs.seg_rows;
    slab = g * ((segs.seg_rows + 127) / 128) + rr / 128;
  } else {
    if (r >= t.end) return -1;
    // the segment holding r: the last one starting at or before it (an empty
    // segment shares its start with the next one)
    int lo = 0, hi = segs.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (t.start[mid] <= r) lo = mid; else hi = mid - 1;
    }
    rr = r - t.start[lo];
    slab = t.cum[lo] + rr / 128;
  }
  const long long cb = (C + 3) / 4;
  return (slab * cb + c / 4) * 512 + (rr % 32) * 16 + ((rr % 128) / 32) * 4 + (c % 4);
}

// -------------------------------------------------------------- row mode
// x: (R, C) contiguous, C % 32 == 0.  q: (R, C) e4m3.  s: scales.
// Each thread handles kUnroll 8-element slots a grid-stride apart and issues
// all their loads before converting, so kUnroll 16-byte loads are in flight.
// kFp4: e2m1 output, packed two per byte (q holds R x C/2 bytes).
template <typename T, bool kFp4 = false>
__global__ void __launch_bounds__(256) quantize_rows_e4m3(const T* __restrict__ x, long long R, long long C,
                                                          uint8_t* __restrict__ q, uint8_t* __restrict__ s,
                                                          int scale_layout, const ScaleSegs segs) {
  constexpr int kUnroll = 4;
  __shared__ SegTable seg_table;
  if (scale_layout == kScaleBlockedSeg && segs.offs) {
    if (threadIdx.x < 32) build_seg_table(seg_table, segs, R);
    __syncthreads();
  }
  const long long total8 = R * C / 8;                  // a multiple of 4: a 32-block never straddles slots
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  const long long SC = C / 32;
  // every lane of a warp runs the same number of iterations (the shuffles
  // need the whole quad), so iterate over warp-rounded ranges
  const long long total8_w = (total8 + 31) / 32 * 32;
  for (long long base = (long long)blockIdx.x * blockDim.x + threadIdx.x; base < total8_w;
       base += kUnroll * stride) {
    float f[kUnroll][8];
    uint32_t m[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = base + u * stride;
      m[u] = 0;
      if (i < total8) {
        load8<T>(x + i * 8, f[u]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[u][k] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int k = 0; k < 8; ++k) m[u] = max(m[u], abs_bits(f[u][k]));
      m[u] = max(m[u], __shfl_xor_sync(0xffffffffu, m[u], 1));
      m[u] = max(m[u], __shfl_xor_sync(0xffffffffu, m[u], 2));
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = base + u * stride;
      if (i >= total8) continue;
      const uint32_t sc = floor_scale(m[u], kFp4 ? 2 : 8);
      const float mult = __uint_as_float((254u - sc) << 23);    // 2^(127 - s)
      if constexpr (kFp4)
        *reinterpret_cast<uint32_t*>(q + i * 4) = e2m1x8(f[u], mult);
      else
        *reinterpret_cast<uint2*>(q + i * 8) = e4m3x8(f[u], mult, m[u]);
      if ((lane & 3) == 0) {
        const long long blk = i / 4;
        if (scale_layout == kScaleRowMajor) {
          s[blk] = (uint8_t)sc;
        } else if (scale_layout == kScaleBlocked) {
          const long long r = blk / SC, c = blk - r * SC;
          s[blocked_sf_offset(r, c, SC)] = (uint8_t)sc;
        } else {
          const long long r = blk / SC, c = blk - r * SC;
          const long long o = blocked_seg_sf_offset(r, c, SC, segs, seg_table);
          if (o >= 0) s[o] = (uint8_t)sc;
        }
      }
    }
  }
}

// ------------------------------------------------------ gathered row mode
// Quantise-on-dispatch: output row i is input row row_index[i] (or zeros
// when row_index[i] is negative -- the padding of a routed group -- or out of
// range), so routing's gather
// and to_mx are one HBM pass.  x (R_in, C) contiguous, C % 32 == 0;
// q (n_rows, C) e4m3; s (n_rows, C/32) row-major.  One thread per 8
// elements, four lanes per 32-block, as quantize_rows_e4m3.
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_gather_e4m3(const T* __restrict__ x,
                                                                 long long in_rows,
                                                                 const int32_t* __restrict__ row_index,
                                                                 long long n_rows, long long C,
                                                                 uint8_t* __restrict__ q, uint8_t* __restrict__ s) {
  const long long per_row = C / 8;
  const long long total8 = n_rows * per_row;
  const long long total8_w = (total8 + 31) / 32 * 32;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total8_w; i += stride) {
    float f[8];
    bool live = false;
    long long r = 0, c8 = 0;
    if (i < total8) {
      r = i / per_row;
      c8 = i - r * per_row;
      const int src = __ldg(row_index + r);
      live = src >= 0 && src < in_rows;   // out-of-range indices read as padding
      if (live) {
        load8<T>(x + (long long)src * C + c8 * 8, f);
      }
    }
    if (!live) {
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = 0.0f;
    }
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) m = max(m, abs_bits(f[k]));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (i >= total8) continue;
    const uint32_t sc = floor_scale(m, 8);
    const float mult = __uint_as_float((254u - sc) << 23);
    *reinterpret_cast<uint2*>(q + i * 8) = e4m3x8(f, mult, m);
    if ((lane & 3) == 0) s[i / 4] = (uint8_t)sc;
  }
}

// -------------------------------------------------------------- col mode
// x: (R, C) contiguous, R % 32 == 0.  Quantises along R and writes the
// transposed result: qt (C, R) e4m3, scales (C, R/32).
// A CTA stages a 32 x 64 tile (32 rows of the block dimension, 64 columns)
// through shared memory so both the reads of x and the writes of qt are
// coalesced.
template <typename T>
__global__ void __launch_bounds__(256) quantize_cols_e4m3(const T* __restrict__ x, long long R, long long C,
                                                          uint8_t* __restrict__ qt, uint8_t* __restrict__ s,
                                                          int scale_layout) {
  __shared__ float tile[32][65];
  const long long RB = R / 32;
  const long long CT = (C + 63) / 64;
  const long long ntiles = RB * CT;
  const int tid = threadIdx.x;
  for (long long t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const long long rb = t / CT, ct = t - rb * CT;
    const long long r0 = rb * 32, c0 = ct * 64;
    // load 32 rows x 64 cols: each thread 8 elements along a row
    {
      const int rr = tid >> 3;          // 0..31
      const int cc = (tid & 7) * 8;     // 0..56
      float f[8];
      if (c0 + cc + 8 <= C) {
        load8<T>(x + (r0 + rr) * C + c0 + cc, f);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = (c0 + cc + k < C) ? to_f32(x[(r0 + rr) * C + c0 + cc + k]) : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) tile[rr][cc + k] = f[k];
    }
    __syncthreads();
    // 64 output rows (columns of x); 4 threads per output row, 8 elements each
    {
      const int oc = tid >> 2;          // 0..63 : column of x = output row
      const int part = tid & 3;         // which 8 of the 32 block elements
      float f[8];
      uint32_t m = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        f[k] = tile[part * 8 + k][oc];
        m = max(m, abs_bits(f[k]));
      }
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
      const long long orow = c0 + oc;
      if (orow < C) {
        const uint32_t sc = floor_scale(m, 8);
        const float mult = __uint_as_float((254u - sc) << 23);
        *reinterpret_cast<uint2*>(qt + orow * R + r0 + part * 8) = e4m3x8(f, mult, m);
        if (part == 0) {
          if (scale_layout == kScaleRowMajor)
            s[orow * RB + rb] = (uint8_t)sc;
          else
            s[blocked_sf_offset(orow, rb, RB)] = (uint8_t)sc;
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace mxgg
