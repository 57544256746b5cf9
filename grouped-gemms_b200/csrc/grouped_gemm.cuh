// Persistent, warp-specialised MXFP8 grouped GEMM for sm_100a.
//
// One kernel body serves the three passes of the MoE layer:
//   * forward / dgrad  (mode kFwd):   out[rows of group g] = A[rows] @ B[g]^T
//     A (M, K) e4m3, B (E, N, K) e4m3, e8m0 scales per 32 along K.
//     Replaces triton_mxfp8_grouped_mm (reference kernels/forward.py:461-606).
//   * wgrad            (mode kWgrad): out[g] = GO_t[:, group g] @ X_t[:, group g]^T
//     GO_t (N, M), X_t (K, M) e4m3, e8m0 scales per 32 tokens; the jagged token
//     range of each group is the contraction.
//     Replaces triton_mxfp8_wgrad (reference kernels/backward.py:217-305).
//
// Work unit = one 128 x BN output tile.  Warp roles (256 threads):
//   warp 0      TMA producer: A and B tiles (128 B swizzle) into a STAGES ring
//   warp 1      MMA issuer: tcgen05.cp of the scales into TMEM, then
//               tcgen05.mma.kind::mxf8f6f4.block_scale (M=128, N=BN, K=32)
//   warps 2-3   scale gatherers (A side, B side): vector loads of the
//               caller's row-major (rows, contraction/32) scales, transposed
//               in registers into the 128x4 scale atom layout tcgen05.cp
//               expects -- no separate re-layout pass over HBM
//   warp 3      also builds the group table in the prologue
//   warps 4-7   epilogue: TMEM -> registers -> bf16/fp32 -> swizzled smem ->
//               TMA store; ragged group edges fall back to predicated stores
//
// Scheduling: a persistent grid (one CTA per SM) walks a device-built
// group->tile map: every CTA reads the group end offsets once, builds the
// per-group start / tile-prefix table in shared memory and decodes tile ids
// with a binary search.  No host synchronisation, no separate routing launch
// (the reference builds a packed map with an extra launch, forward.py:340-365).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace mxgg {

constexpr int kBM = 128;          // tile rows (MMA M)
constexpr int kBK = 128;          // contraction elements per stage (= one 128 B swizzle row of e4m3)
constexpr int kThreads = 256;
constexpr int kMaxGroups = 256;   // groups handled by the in-kernel table
constexpr int kTmemCols = 512;

enum : int { kFwd = 0, kWgrad = 1 };
enum : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2 };

// error bits written to GemmParams::status
enum : uint32_t {
  kErrProducerWait = 1u,
  kErrScaleWait = 2u,
  kErrMmaWait = 4u,
  kErrAccWait = 8u,
  kErrEpilogueWait = 16u,
  kErrDrain = 32u,
};

struct GemmParams {
  int mode;
  int E;
  int M, N, K;               // fwd: out (M,N), contraction K.  wgrad: out (E,N,K), contraction = tokens M
  int rows_a, rows_b;        // rows of the A / B operand tensors (for clamping scale reads)
  int contraction;           // fwd: K, wgrad: M
  const int32_t* offs;       // (E,) cumulative group ends
  const uint8_t* sfa;        // A scales, row-major (rows_a, contraction/32)
  const uint8_t* sfb;        // B scales, row-major (rows_b, contraction/32)
  long long sf_ld;           // bytes per scale row (= contraction/32)
  void* out;
  long long out_ld;          // elements per output row
  long long out_rows;        // rows of the output tensor
  int out_cols;              // valid output columns (fwd: N, wgrad: K)
  int sf_vec;                // scale gather width in 4-byte words (4, 2, 1), 0 = byte gathers
  int tma_store;             // 1: output rows are 16-byte aligned for TMA stores
  int group_m;               // rasterisation band (m-tiles) for the forward pass
  uint32_t* status;          // error word (device memory), 0 = ok
};

struct Unit {
  int a_row;         // TMA row of the A tile
  int b_row;         // TMA row of the B tile
  long long out_row; // output row of tile row 0
  int out_col;       // output column of tile column 0
  int valid_rows;    // rows of the tile owned by this unit (0..128)
  int st_begin;      // first 128-element contraction stage (global index)
  int st_count;      // number of stages (0 = the output tile is all zeros)
  int c_begin;       // contraction range [c_begin, c_end), multiples of 32
  int c_end;
};

template <int BN, int STAGES, typename OutT>
struct SmemLayout {
  static constexpr int kEpiCols = 64 / sizeof(OutT);   // 64-byte staging rows
  alignas(1024) uint8_t a[STAGES][kBM * kBK];
  alignas(1024) uint8_t b[STAGES][BN * kBK];
  alignas(1024) uint8_t epi[4][2][32 * 64];            // per epilogue warp, double buffered
  alignas(16) uint8_t sfa[STAGES][kBM * 4];
  alignas(16) uint8_t sfb[STAGES][BN * 4];
  alignas(8) uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int num_units;
  int g_start[kMaxGroups];
  int g_end[kMaxGroups];
  int g_cum[kMaxGroups + 1];
};

__device__ __forceinline__ int cdiv_i(int a, int b) { return (a + b - 1) / b; }

// Group table: start/end rows (fwd) or token ranges (wgrad) per group and an
// exclusive prefix of m-tiles.  Offsets are clamped into [0, R] and made
// monotone so that out-of-range or decreasing offsets can never address memory
// outside the operands.
template <class S>
__device__ __forceinline__ void build_group_table(S* sm, const GemmParams& p, int R) {
  const int lane = ptx::lane_id();
  int carry_max = 0, carry_sum = 0;
  for (int base = 0; base < p.E; base += 32) {
    const int i = base + lane;
    int c = 0;
    if (i < p.E) c = min(max(__ldg(p.offs + i), 0), R);
    int v = (i < p.E) ? max(c, carry_max) : carry_max;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v = max(v, u);
    }
    int prev = __shfl_up_sync(0xffffffffu, v, 1);
    if (lane == 0) prev = carry_max;
    const int start = prev, end = v;
    int t = (i < p.E) ? cdiv_i(end - start, kBM) : 0;
    int incl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (i < p.E) {
      sm->g_start[i] = start;
      sm->g_end[i] = end;
      sm->g_cum[i] = carry_sum + incl - t;
    }
    carry_max = __shfl_sync(0xffffffffu, v, 31);
    carry_sum += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) sm->g_cum[p.E] = carry_sum;
}

template <int BN, class S>
__device__ __forceinline__ Unit decode_unit(const S* sm, const GemmParams& p, int t) {
  Unit u;
  if (p.mode == kFwd) {
    const int NT = cdiv_i(p.N, BN);
    const int MT = sm->g_cum[p.E];
    const int gm = p.group_m;
    const int band = t / (gm * NT);
    const int r = t - band * gm * NT;
    const int m0 = band * gm;
    const int gsz = min(gm, MT - m0);
    const int n = r / gsz;
    const int m = m0 + (r - n * gsz);
    // group owning global m-tile m: last g with g_cum[g] <= m
    int lo = 0, hi = p.E - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sm->g_cum[mid] <= m) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int row0 = sm->g_start[g] + (m - sm->g_cum[g]) * kBM;
    u.a_row = row0;
    u.b_row = g * p.N + n * BN;
    u.out_row = row0;
    u.out_col = n * BN;
    u.valid_rows = min(kBM, sm->g_end[g] - row0);
    u.st_begin = 0;
    u.st_count = cdiv_i(p.K, kBK);
    u.c_begin = 0;
    u.c_end = p.K;
  } else {
    const int NT = cdiv_i(p.N, kBM);
    const int KT = cdiv_i(p.K, BN);
    const int g = t / (NT * KT);
    const int r = t - g * NT * KT;
    const int nt = r / KT;
    const int kt = r - nt * KT;
    const int s = sm->g_start[g], e = sm->g_end[g];
    u.a_row = nt * kBM;
    u.b_row = kt * BN;
    u.out_row = (long long)g * p.N + nt * kBM;
    u.out_col = kt * BN;
    u.valid_rows = min(kBM, p.N - nt * kBM);
    if (e > s) {
      u.st_begin = s / kBK;
      u.st_count = cdiv_i(e, kBK) - u.st_begin;
    } else {
      u.st_begin = 0;
      u.st_count = 0;
    }
    u.c_begin = s;
    u.c_end = e;
  }
  return u;
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void raise_error(const GemmParams& p, volatile int* abort, uint32_t code) {
  atomicOr(p.status, code);
  *abort = 1;
}

template <int BN, int STAGES, int ACC, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  static_assert(BN % 128 == 0 && BN <= 256, "BN must be 128 or 256");
  static_assert(ACC * BN + 2 * (4 + BN / 32) <= kTmemCols, "tensor memory budget");
  using S = SmemLayout<BN, STAGES, OutT>;
  constexpr int kEpiCols = S::kEpiCols;
  constexpr int kSfaCol = ACC * BN;            // two scale buffers follow the accumulators
  constexpr uint32_t kSfCols = 4 + BN / 32;
  constexpr uint32_t kStageBytes = (kBM + BN) * kBK;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  S* sm = reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort = &sm->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ------------------------------------------------------------ prologue
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(ptx::smem_u32(&sm->full[s]), 3);   // TMA producer + two scale gatherers
      ptx::mbar_init(ptx::smem_u32(&sm->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(ptx::smem_u32(&sm->tfull[a]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm->tempty[a]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(&sm->drain), 1);
    sm->abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(&sm->tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 3) {
    build_group_table(sm, p, p.M);   // fwd: rows of A; wgrad: tokens
    __syncwarp();
    if (lane == 0) {
      if (p.mode == kFwd)
        sm->num_units = sm->g_cum[p.E] * cdiv_i(p.N, BN);
      else
        sm->num_units = p.E * cdiv_i(p.N, kBM) * cdiv_i(p.K, BN);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  const uint32_t tmem_base = sm->tmem_base;
  const int num_units = sm->num_units;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_units && ok; t += gridDim.x) {
        const Unit u = decode_unit<BN>(sm, p, t);
        for (int s = 0; s < u.st_count; ++s, ++it) {
          const int stage = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!ptx::mbar_wait(ptx::smem_u32(&sm->empty[stage]), ph ^ 1u, abort)) {
            raise_error(p, abort, kErrProducerWait);
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&sm->full[stage]);
          ptx::mbar_arrive_expect_tx(fb, kStageBytes);
          const int x = (u.st_begin + s) * kBK;
          ptx::tma_load_2d(ptx::smem_u32(sm->a[stage]), &tmap_a, fb, x, u.a_row);
          ptx::tma_load_2d(ptx::smem_u32(sm->b[stage]), &tmap_b, fb, x, u.b_row);
        }
      }
      if (!ok || *abort) {
        // Error path: give loads already in flight up to 50 ms to land before
        // the CTA retires (their barrier may never complete if a peer role
        // stopped early, so this wait is bounded by time, not by the barrier).
        const uint32_t issued = it;
        for (uint32_t k = (issued > STAGES ? issued - STAGES : 0); k < issued; ++k) {
          const uint64_t t0 = ptx::globaltimer();
          while (!ptx::mbar_try_wait(ptx::smem_u32(&sm->full[k % STAGES]), (k / STAGES) & 1u)) {
            if (ptx::globaltimer() - t0 > 50000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = ptx::idesc_mxf8(kBM, BN, 0, 0);
      constexpr uint32_t kAStep = (kBM * kBK) >> 4;     // descriptor start-address step per stage
      constexpr uint32_t kBStep = (BN * kBK) >> 4;
      const uint64_t adesc0 = ptx::kmajor_sw128_desc(ptx::smem_u32(sm->a[0]));
      const uint64_t bdesc0 = ptx::kmajor_sw128_desc(ptx::smem_u32(sm->b[0]));
      const uint64_t sfadesc0 = ptx::sf_copy_desc(ptx::smem_u32(sm->sfa[0]));
      const uint64_t sfbdesc0 = ptx::sf_copy_desc(ptx::smem_u32(sm->sfb[0]));
      uint32_t it = 0, ai = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_units && ok; t += gridDim.x, ++ai) {
        const Unit u = decode_unit<BN>(sm, p, t);
        const int acc = ai % ACC;
        const uint32_t aph = (ai / ACC) & 1u;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm->tempty[acc]), aph ^ 1u, abort)) {
          raise_error(p, abort, kErrAccWait);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        uint32_t accumulate = 0;
        for (int s = 0; s < u.st_count; ++s, ++it) {
          const uint32_t stage = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!ptx::mbar_wait(ptx::smem_u32(&sm->full[stage]), ph, abort)) {
            raise_error(p, abort, kErrMmaWait);
            ok = false;
            break;
          }
          // scale factors of this stage -> TMEM (double-buffered so the copy
          // never waits on the previous stage's MMAs)
          const uint32_t sfa_t = tmem_base + kSfaCol + (it & 1u) * kSfCols;
          const uint32_t sfb_t = sfa_t + 4;
          ptx::tc_cp_32x128b_warpx4(sfa_t, sfadesc0 + (uint64_t)(stage * ((kBM * 4) >> 4)));
#pragma unroll
          for (int b = 0; b < BN / 128; ++b)
            ptx::tc_cp_32x128b_warpx4(sfb_t + 4 * b, sfbdesc0 + (uint64_t)(stage * ((BN * 4) >> 4) + b * (512 >> 4)));
          const uint64_t adesc = adesc0 + (uint64_t)(stage * kAStep);
          const uint64_t bdesc = bdesc0 + (uint64_t)(stage * kBStep);
          const int base = (u.st_begin + s) * kBK;
          const int j0 = max(0, (u.c_begin - base) / 32);
          const int j1 = min(4, (u.c_end - base + 31) / 32);
          if (j0 == 0 && j1 == 4) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              ptx::tc_mma_mxf8(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j),
                               ptx::idesc_with_sf(kIdesc, j, j), sfa_t | (uint32_t(j) << 30),
                               sfb_t | (uint32_t(j) << 30), (j == 0) ? accumulate : 1u);
            }
            accumulate = 1;
          } else {
            for (int j = j0; j < j1; ++j) {
              ptx::tc_mma_mxf8(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j),
                               ptx::idesc_with_sf(kIdesc, j, j), sfa_t | (uint32_t(j) << 30),
                               sfb_t | (uint32_t(j) << 30), accumulate);
              accumulate = 1;
            }
          }
          ptx::tc_commit(ptx::smem_u32(&sm->empty[stage]));
        }
        if (!ok) break;
        ptx::tc_commit(ptx::smem_u32(&sm->tfull[acc]));
      }
      // every MMA this thread issued has retired before TMEM is released
      ptx::tc_commit(ptx::smem_u32(&sm->drain));
      volatile int never = 0;
      if (!ptx::mbar_wait(ptx::smem_u32(&sm->drain), 0, &never)) atomicOr(p.status, kErrDrain);
    }
  } else if (warp == 2 || warp == 3) {
    // -------------------------------------------------------- scale gather
    // Warp 2 gathers the A-side scales, warp 3 the B-side ones, from the
    // caller's row-major (rows, contraction/32) layout into the 128x4 atom
    // layout tcgen05.cp reads: atom byte (r % 32) * 16 + (r / 32) * 4 + k.
    // Lane l owns rows l + 32 i; one vector load per row fetches the scales of
    // kVec consecutive stages, and a register transpose turns four rows into
    // the lane's 16-byte atom row.  Each stage is fenced into the async proxy
    // by the writers and published with one arrive, so the MMA thread never
    // fences.
    const bool side_a = (warp == 2);
    constexpr int kMaxRows = BN / 32;                 // rows per lane on the B side (A side: 4)
    const int nrows_lane = side_a ? 4 : kMaxRows;
    const uint8_t* sf = side_a ? p.sfa : p.sfb;
    const int rows_total = side_a ? p.rows_a : p.rows_b;
    const int vec = p.sf_vec;                        // words per load: 4, 2, 1; 0 = byte gathers
    const int G = vec > 0 ? vec : 1;                 // stages per load
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_units && ok; t += gridDim.x) {
      const Unit u = decode_unit<BN>(sm, p, t);
      const int rbase = side_a ? u.a_row : u.b_row;
      const uint8_t* rowp[kMaxRows];
#pragma unroll
      for (int i = 0; i < kMaxRows; ++i) {
        const int row = min(max(rbase + lane + 32 * i, 0), rows_total - 1);
        rowp[i] = sf + (long long)row * p.sf_ld;
      }
      int s = 0;
      while (s < u.st_count && ok) {
        const int st0 = u.st_begin + s;
        const int cst = st0 - st0 % G;               // first stage of the loaded chunk
        const int cend = min(cst + G, u.st_begin + u.st_count);
        uint32_t w[kMaxRows][4];
#pragma unroll
        for (int i = 0; i < kMaxRows; ++i) {
          if (i < nrows_lane) {
            const uint8_t* q = rowp[i] + 4LL * cst;
            if (vec == 4) {
              const uint4 v = __ldg(reinterpret_cast<const uint4*>(q));
              w[i][0] = v.x; w[i][1] = v.y; w[i][2] = v.z; w[i][3] = v.w;
            } else if (vec == 2) {
              const uint2 v = __ldg(reinterpret_cast<const uint2*>(q));
              w[i][0] = v.x; w[i][1] = v.y; w[i][2] = 0; w[i][3] = 0;
            } else if (vec == 1) {
              w[i][0] = __ldg(reinterpret_cast<const uint32_t*>(q)); w[i][1] = w[i][2] = w[i][3] = 0;
            } else {
              uint32_t x = 0;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const long long cc = 4LL * cst + j;
                const uint32_t b = (cc < p.sf_ld) ? (uint32_t)__ldg(rowp[i] + cc) : 127u;
                x |= b << (8 * j);
              }
              w[i][0] = x; w[i][1] = w[i][2] = w[i][3] = 0;
            }
          }
        }
        for (int st = st0; st < cend; ++st, ++s, ++it) {
          const int stage = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!ptx::mbar_wait(ptx::smem_u32(&sm->empty[stage]), ph ^ 1u, abort)) {
            raise_error(p, abort, kErrScaleWait);
            ok = false;
            break;
          }
          const int wi = st - cst;
          const uint32_t dst = (side_a ? ptx::smem_u32(sm->sfa[stage]) : ptx::smem_u32(sm->sfb[stage])) + lane * 16;
#pragma unroll
          for (int a = 0; a < kMaxRows / 4; ++a) {
            if (4 * a < nrows_lane) {
              uint32_t x[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const uint32_t* r = w[4 * a + c];
                x[c] = (wi == 0) ? r[0] : (wi == 1) ? r[1] : (wi == 2) ? r[2] : r[3];
              }
              asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + 512 * a), "r"(x[0]), "r"(x[1]),
                           "r"(x[2]), "r"(x[3])
                           : "memory");
            }
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&sm->full[stage]));
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    uint32_t ai = 0;
    int buf = 0;
    for (int t = blockIdx.x; t < num_units; t += gridDim.x, ++ai) {
      const Unit u = decode_unit<BN>(sm, p, t);
      const int acc = ai % ACC;
      const uint32_t aph = (ai / ACC) & 1u;
      if (!ptx::mbar_wait(ptx::smem_u32(&sm->tfull[acc]), aph, abort)) {
        raise_error(p, abort, kErrEpilogueWait);
        break;
      }
      ptx::tc_fence_after();
      const int rows_here = min(max(u.valid_rows - 32 * q, 0), 32);
      const bool use_tma = p.tma_store && rows_here == 32;
      const bool zero = (u.st_count == 0);
      const uint32_t t_row = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
      const long long grow = u.out_row + 32 * q + lane;   // this thread's output row
#pragma unroll 1
      for (int c = 0; c < BN / kEpiCols; ++c) {
        uint32_t v[kEpiCols];
        if (!zero) {
          if constexpr (kEpiCols == 32) {
            ptx::tmem_ld_32x32b_x32(t_row + c * kEpiCols, reinterpret_cast<uint32_t(&)[32]>(v));
          } else {
            ptx::tmem_ld_32x32b_x16(t_row + c * kEpiCols, reinterpret_cast<uint32_t(&)[16]>(v));
          }
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < kEpiCols; ++i) v[i] = 0u;
        }
        if (c == BN / kEpiCols - 1) {
          // accumulator fully read: hand it back to the MMA warp
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&sm->tempty[acc]));
        }
        if (rows_here == 0) continue;
        const int col0 = u.out_col + c * kEpiCols;
        if (col0 >= p.out_cols) continue;
        // 64 output bytes for this thread's row
        uint32_t w[16];
        if constexpr (sizeof(OutT) == 4) {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = v[i];
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack2<OutT>(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        }
        if (use_tma) {
          uint8_t* stg = sm->epi[q][buf];
          if (lane == 0) ptx::bulk_wait_read<1>();   // the store that last used this buffer has read it
          __syncwarp();
          const uint32_t row_base = ptx::smem_u32(stg) + lane * 64;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t chunk = (uint32_t)(j ^ ((lane >> 1) & 3));   // 64 B swizzle
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + chunk * 16),
                         "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                         : "memory");
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(&tmap_out, ptx::smem_u32(stg), col0, (int)(u.out_row + 32 * q));
            ptx::bulk_commit();
          }
          buf ^= 1;
        } else if (lane < rows_here && grow < p.out_rows) {
          OutT* dst = reinterpret_cast<OutT*>(p.out) + grow * p.out_ld + col0;
          const int ncols = min(kEpiCols, p.out_cols - col0);
          if (ncols == kEpiCols && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
            uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
            for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          } else if constexpr (sizeof(OutT) == 4) {
            uint32_t* d = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j < ncols) d[j] = w[j];
          } else {
            uint16_t* d = reinterpret_cast<uint16_t*>(dst);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) d[j] = (uint16_t)(w[j >> 1] >> ((j & 1) * 16));
          }
        }
      }
    }
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace mxgg
