// Scale-factor packing for the block-scaled grouped GEMM.
//
// The reference's callers hand over e8m0 scales row-major, (rows,
// contraction/32) (utils.to_mx, utils.py:67-105).  The GEMM's scale writers
// read them in the blocked layout: per 128-row slab and per 128-element
// contraction stage one 512-byte atom, byte (r % 32) * 16 + (r / 32) * 4 + k
// for row r of the slab and k-block k of the stage -- lane r % 32 of the atom
// is the 16 bytes TMEM lane r % 32 of every quarter holds in the block-scaled
// MMA's scale layout.  Atoms are stored [slab][stage][512 B], slabs in order:
//
//   forward / dgrad A   each group's rows in 128-row slabs, a new slab at
//                       every group start (group g's slabs follow those of
//                       groups 0 .. g-1)
//   forward / dgrad B   ceil(N / 128) slabs per expert
//   wgrad A and B       ceil(rows / 128) slabs over the whole operand
//
// This is torch's blocked scale layout for grouped MXFP8 GEMMs (to_blocked of
// each group's / expert's scale rows, concatenated); it depends on neither
// the tile shape nor the schedule, so a quantiser can write it once
// (mxgg_quantize_mx's blocked modes) and the GEMM takes it as is.  This pass
// converts row-major scales into it (the reference instead re-lays scales on
// the host for every call, forward.py:537-561).  Rows past the operand are
// clamped: their scales only feed output rows that are never stored.
#pragma once

#include <cstdint>

#include "grouped_gemm.cuh"

namespace mxgg {

struct PackParams {
  int mode;              // kFwd / kWgrad
  int E;                 // fwd: groups of A rows
  int stages;            // ceil(contraction / 128)
  const int32_t* offs;   // fwd: group end offsets of the A rows
  const uint8_t* sfa;    // (rows_a, sf_ld) row-major
  const uint8_t* sfb;    // (rows_b, sf_ld) row-major
  int rows_a, rows_b;
  long long sf_ld;       // bytes per scale row
  int vec;               // 4: 16-byte row loads are aligned, 1: 4-byte, 0: bytes
  int a_slabs;           // A slabs to write (fwd: an upper bound; slabs past the groups' are skipped)
  int b_slabs;           // B slabs to write
  int b_height;          // rows per B matrix (fwd: N, one matrix per expert; wgrad: K)
  uint8_t* a_out;
  uint8_t* b_out;
  int* zero;             // split-tail arrival counters to clear (or null)
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
        const uint32_t v = (cc < p.sf_ld) ? (uint32_t)__ldg(row + cc) : 0u;
        x |= v << (8 * b);
      }
      w[j] = x;
    }
  }
}

// One warp per (128-row slab, 4-stage chunk).  Lane l owns rows l + 32 c of
// the slab; a register transpose turns its four rows into the 16-byte atom
// row it writes for each stage, so every atom store is a coalesced 512 B.
// bx / nbx: this block's index among the blocks that share the work.
__device__ __forceinline__ void pack_scales_body(const PackParams& p, unsigned bx, unsigned nbx) {
  __shared__ int s_start[kMaxGroups];
  __shared__ int s_cum[kMaxGroups + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The GEMM that follows may launch now: its prologue and first tile loads
  // need nothing from this kernel, and the roles that read the atoms and
  // counters written here wait for this grid to finish (griddepcontrol.wait).
  ptx::griddep_launch_dependents();
  if (p.mode == kFwd && p.a_slabs > 0) {
    if (warp == 0) {
      // the GEMM's group table: clamped, monotone starts; 128-row slab prefix
      int carry_max = 0, carry_sum = 0;
      for (int base = 0; base < p.E; base += 32) {
        const int i = base + lane;
        int c = 0;
        if (i < p.E) c = min(max(__ldg(p.offs + i), 0), p.rows_a);
        int v = (i < p.E) ? max(c, carry_max) : carry_max;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v = max(v, u);
        }
        int prev = __shfl_up_sync(0xffffffffu, v, 1);
        if (lane == 0) prev = carry_max;
        int t = (i < p.E) ? cdiv_i(v - prev, 128) : 0;
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
    for (long long i = (long long)bx * blockDim.x + threadIdx.x; i < p.zero_count; i += (long long)nbx * blockDim.x)
      p.zero[i] = 0;
  }
  const int chunks = (p.stages + 3) / 4;
  const long long a_work = (long long)p.a_slabs * chunks;
  const long long b_work = (long long)p.b_slabs * chunks;
  const int nb = cdiv_i(max(p.b_height, 1), 128);
  const long long nwarps = (long long)nbx * (blockDim.x >> 5);
  for (long long wi = (long long)bx * (blockDim.x >> 5) + warp; wi < a_work + b_work; wi += nwarps) {
    const bool side_a = wi < a_work;
    const long long idx = side_a ? wi : wi - a_work;
    const int q = (int)(idx % chunks);
    const int slab = (int)(idx / chunks);
    long long row0;
    const uint8_t* sf;
    int rows_total;
    if (side_a) {
      sf = p.sfa;
      rows_total = p.rows_a;
      if (p.mode == kFwd) {
        if (slab >= s_cum[p.E]) continue;   // beyond the slabs of this call's groups
        int lo = 0, hi = p.E - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_cum[mid] <= slab) lo = mid; else hi = mid - 1;
        }
        row0 = (long long)s_start[lo] + 128LL * (slab - s_cum[lo]);
      } else {
        row0 = 128LL * slab;
      }
    } else {
      sf = p.sfb;
      rows_total = p.rows_b;
      row0 = (long long)(slab / nb) * p.b_height + 128LL * (slab % nb);
    }
    uint8_t* dst0 = (side_a ? p.a_out : p.b_out) + (long long)slab * p.stages * 512;
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
        uint4* d = reinterpret_cast<uint4*>(dst0 + (long long)st * 512 + lane * 16);
        *d = make_uint4(w[0][j], w[1][j], w[2][j], w[3][j]);
      }
    }
  }
}

__global__ void __launch_bounds__(256) pack_scales_kernel(const PackParams p) {
  pack_scales_body(p, blockIdx.x, gridDim.x);
}

// Several forward-A packs in one launch (an expert-parallel sender packing
// its rows' scales for every destination): blockIdx.y picks the pack.
struct PackMulti {
  PackParams p[kMaxDst];
};

__global__ void __launch_bounds__(256) pack_scales_multi_kernel(const PackMulti m) {
  pack_scales_body(m.p[blockIdx.y], blockIdx.x, gridDim.x);
}

}  // namespace mxgg
