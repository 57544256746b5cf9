// Scale-factor packing for the block-scaled grouped GEMM.
//
// The reference's callers hand over e8m0 scales row-major, (rows,
// contraction/32) (utils.to_mx, utils.py:67-105).  The GEMM's scale writers
// want, per 128-row slab and per 128-element contraction stage, one 512-byte
// atom laid out as byte (r % 32) * 16 + (r / 32) * 4 + k (row r, k-block k):
// lane r % 32 of the atom is the 16 bytes that TMEM lane r % 32 of every
// quarter holds in the block-scaled MMA's scale layout.  This pass
// writes exactly the atoms the GEMM will read, in the order it reads them, so
// the GEMM's producer can fetch a stage's scales with one TMA load each
// (instead of the reference's per-call host re-layout, forward.py:537-561):
//
//   A side  [sub-tile][stage][512 B]        sub-tile = 128 rows of a tile
//   B side  [tile][stage][BN/128][512 B]    all BN rows of an n-tile
//
// Forward tiles follow the group boundaries (a tile never spans two groups),
// so the A-side sub-tile of (group g, tile mt, half h) starts at row
// start_g + mt * tile_m + 128 h.  Rows past the operand are clamped: their
// scales only feed output rows that are never stored.
#pragma once

#include <cstdint>

#include "grouped_gemm.cuh"

namespace mxgg {

struct PackParams {
  int mode;              // kFwd / kWgrad
  int E;
  int M, N, K;           // as GemmParams
  int tile_m;            // 128 * PAIR
  int tile_n;            // BN
  int stages;            // ceil(contraction / 128)
  const int32_t* offs;
  const uint8_t* sfa;    // (rows_a, sf_ld) row-major
  const uint8_t* sfb;    // (rows_b, sf_ld) row-major
  int rows_a, rows_b;
  long long sf_ld;       // bytes per scale row
  int vec;               // 4: 16-byte row loads are aligned, 1: 4-byte, 0: bytes
  int a_subtiles;        // A-side sub-tiles provisioned in the workspace
  int b_tiles;           // B-side tiles (fwd: experts x n-tiles)
  uint8_t* a_out;
  uint8_t* b_out;
  int* zero;             // stream-K arrival counters to clear (or null)
  long long zero_count;
};

// Load the scale words of stages [q*4, q*4+4) for one row: word j = the four
// k-blocks of stage q*4 + j.
__device__ __forceinline__ void load_row_words(const uint8_t* row, const PackParams& p, int q, uint32_t (&w)[4]) {
  const long long c0 = 16LL * q;
  if (p.vec == 4 && 4 * q + 3 < p.stages) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + c0));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    return;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const long long cw = c0 + 4 * j;
    if (p.vec >= 1 && cw + 4 <= p.sf_ld) {
      w[j] = __ldg(reinterpret_cast<const uint32_t*>(row + cw));
    } else {
      uint32_t x = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const long long cc = cw + b;
        const uint32_t v = (cc < p.sf_ld) ? (uint32_t)__ldg(row + cc) : 127u;
        x |= v << (8 * b);
      }
      w[j] = x;
    }
  }
}

// One warp per (128-row slab, 4-stage chunk).  Lane l owns rows l + 32 c of
// the slab; a register transpose turns its four rows into the 16-byte atom
// row it writes for each stage, so every atom store is a coalesced 512 B.
__global__ void __launch_bounds__(256) pack_scales_kernel(const PackParams p) {
  __shared__ int s_start[kMaxGroups];
  __shared__ int s_cum[kMaxGroups + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The GEMM that follows may launch now: its prologue and first tile loads
  // need nothing from this kernel, and the roles that read the atoms and
  // counters written here wait for this grid to finish (griddepcontrol.wait).
  ptx::griddep_launch_dependents();
  if (p.mode == kFwd) {
    if (warp == 0) {
      // same group table as the GEMM: clamped, monotone starts; tile prefix
      int carry_max = 0, carry_sum = 0;
      for (int base = 0; base < p.E; base += 32) {
        const int i = base + lane;
        int c = 0;
        if (i < p.E) c = min(max(__ldg(p.offs + i), 0), p.M);
        int v = (i < p.E) ? max(c, carry_max) : carry_max;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v = max(v, u);
        }
        int prev = __shfl_up_sync(0xffffffffu, v, 1);
        if (lane == 0) prev = carry_max;
        int t = (i < p.E) ? cdiv_i(v - prev, p.tile_m) : 0;
        int incl = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int u = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += u;
        }
        if (i < p.E) {
          s_start[i] = prev;
          s_cum[i] = carry_sum + incl - t;
        }
        carry_max = __shfl_sync(0xffffffffu, v, 31);
        carry_sum += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) s_cum[p.E] = carry_sum;
    }
    __syncthreads();
  }
  if (p.zero) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < p.zero_count;
         i += (long long)gridDim.x * blockDim.x)
      p.zero[i] = 0;
  }
  const int halves = p.tile_m / 128;
  const int bsub = p.tile_n / 128;
  const int chunks = (p.stages + 3) / 4;
  const int a_work = p.a_subtiles * chunks;
  const int b_work = p.b_tiles * bsub * chunks;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int wi = blockIdx.x * (blockDim.x >> 5) + warp; wi < a_work + b_work; wi += nwarps) {
    const bool side_a = wi < a_work;
    const int idx = side_a ? wi : wi - a_work;
    const int q = idx % chunks;
    const int slab = idx / chunks;      // A: sub-tile; B: tile * bsub + b
    long long row0;
    const uint8_t* sf;
    int rows_total;
    uint8_t* dst0;
    long long dst_stage_stride;
    if (side_a) {
      sf = p.sfa;
      rows_total = p.rows_a;
      const int m = slab / halves, h = slab % halves;
      if (p.mode == kFwd) {
        if (m >= s_cum[p.E]) continue;   // beyond the tiles this call produces
        int lo = 0, hi = p.E - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_cum[mid] <= m) lo = mid; else hi = mid - 1;
        }
        row0 = (long long)s_start[lo] + (long long)(m - s_cum[lo]) * p.tile_m + 128LL * h;
      } else {
        row0 = 128LL * slab;
      }
      dst0 = p.a_out + (long long)slab * p.stages * 512;
      dst_stage_stride = 512;
    } else {
      sf = p.sfb;
      rows_total = p.rows_b;
      const int tile = slab / bsub, b = slab % bsub;
      if (p.mode == kFwd) {
        const int NT = cdiv_i(p.N, p.tile_n);
        const int g = tile / NT, nt = tile % NT;
        row0 = (long long)g * p.N + (long long)nt * p.tile_n + 128LL * b;
      } else {
        row0 = (long long)tile * p.tile_n + 128LL * b;
      }
      dst0 = p.b_out + ((long long)tile * p.stages * bsub + b) * 512;
      dst_stage_stride = 512LL * bsub;
    }
    uint32_t w[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const long long r = min(max(row0 + lane + 32 * c, 0LL), (long long)rows_total - 1);
      load_row_words(sf + r * p.sf_ld, p, q, w[c]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int st = 4 * q + j;
      if (st < p.stages) {
        uint4* d = reinterpret_cast<uint4*>(dst0 + (long long)st * dst_stage_stride + lane * 16);
        *d = make_uint4(w[0][j], w[1][j], w[2][j], w[3][j]);
      }
    }
  }
}

}  // namespace mxgg
