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
// Work unit = one (128 * PAIR) x BN output tile.  With PAIR == 2 a cluster of
// two CTAs on neighbouring SMs computes a 256-row tile with one
// tcgen05.mma.cta_group::2 stream: each CTA stages its own 128 rows of A and
// half of the BN rows of B (plain TMA loads, no multicast), so every byte a
// CTA pulls from L2 feeds twice the MMA work of a single-CTA tile.
//
// Warp roles (320 threads per CTA):
//   warps 0-3   scale writers: per stage, the CTA's scale atoms (pre-packed by
//               pack_scales_kernel) go from global memory, through a register
//               ring loaded kSfRing stages ahead, to a ring of kSfSlots scale
//               slots in TMEM with tcgen05.st, warp q writing its own 32-lane
//               quarter (the block-scaled MMA reads the same 32-row atom from
//               every quarter); then they arrive on the stage's full barrier.
//               Moving the scales with tcgen05.cp instead puts three copies
//               per stage into the tensor pipe's instruction stream, where
//               they cost ~135 of a stage's ~490 MMA cycles (measured on
//               B200); tcgen05.st from other warps leaves the pipe to the
//               MMAs.  Warp 3 also builds the group table in the prologue.
//   warps 4-7   epilogue: TMEM -> registers -> bf16/fp32 -> swizzled smem ->
//               TMA store; ragged group edges fall back to predicated stores;
//               on request also the MX-quantised rows and transpose (to_mx and
//               to_mx_dim1 of the output) from the same registers
//   warp 8      TMA producer: per stage the A and B tiles (128 B swizzle) into
//               a STAGES ring on one transaction barrier (the pair's leader
//               counts both CTAs' bytes and the scale writers' arrivals)
//   warp 9      MMA issuer (the leader CTA's lane 0): one wait per stage (its
//               full barrier), four tcgen05.mma.kind::mxf8f6f4.block_scale
//               (K=32), one commit.  A second per-stage wait, on a barrier of
//               the scale writers' own, measured ~10 % slower.
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
#include "quantize.cuh"

namespace mxgg {

constexpr int kBM = 128;          // rows per CTA (MMA M per CTA)
constexpr int kBK = 128;          // contraction elements per stage (= one 128 B swizzle row of e4m3)
constexpr int kSfWarp0 = 0;       // scale writers: warps 0-3
constexpr int kEpiWarp0 = 4;      // epilogue: warps 4-7
constexpr int kProdWarp = 8;      // TMA producer
constexpr int kMmaWarp = 9;       // MMA issuer
constexpr int kThreads = 320;
constexpr int kSfSlotsMax = 5;    // scale slots in TMEM (stages the writers may run ahead), at most
constexpr int kSfRing = 4;        // stages of scale atoms the writers hold in registers
constexpr int kMaxGroups = 256;   // groups handled by the in-kernel table
constexpr int kMaxDst = 8;        // output destinations (ranks) of an expert-parallel forward
constexpr int kMaxSrc = 32;       // source ids of a streamed dispatch (bits of a readiness mask)
constexpr int kTmemCols = 512;

enum : int { kFwd = 0, kWgrad = 1 };

// Optional paths of the GEMM kernel, compiled into a build only when its
// calls need them (a build's template argument kFeat is a mask of these):
enum : int {
  kFeatSplit = 1,   // split-tail schedule: pieces, fp32 partials, their reduction
  kFeatEp = 2,      // expert parallel: peer outputs and inboxes, streamed sources, rows read in place
  kFeatQuant = 4,   // MX-quantised outputs (rows and transposed) from the epilogue
  kFeatAcc = 8,     // accumulate into an fp32 output
};

// error bits written to GemmParams::status
enum : uint32_t {
  kErrProducerWait = 1u,
  kErrScaleWait = 2u,
  kErrMmaWait = 4u,
  kErrAccWait = 8u,
  kErrEpilogueWait = 16u,
  kErrDrain = 32u,
  // 64 is the cross-GPU barrier's (peer.cuh)
  kErrSourceWait = 128u,     // expert parallel: a source's rows never arrived
  kErrQtRows = 256u,         // transposed quantised output: a group not on the 32-row grid
};

struct GemmParams {
  int mode;
  int E;
  int M, N, K;               // fwd: out (M,N), contraction K.  wgrad: out (E,N,K), contraction = tokens M
  int rows_a, rows_b;        // rows of the A / B operand tensors (for clamping scale reads)
  int contraction;           // fwd: K, wgrad: M
  const int32_t* offs;       // (E,) cumulative group ends
  const int32_t* group_expert;  // fwd: expert (B slice) of each group, or null for group g -> expert g
  int n_experts;             // fwd: experts in B (E when group_expert is null)
  int b_fmt;                 // B element type in the MMA's encoding: 0 e4m3, 5 e2m1 (TMA-unpacked to 8-bit slots)
  void* out;
  long long out_ld;          // elements per output row
  long long out_rows;        // rows of the output tensor
  int out_cols;              // valid output columns (fwd: N, wgrad: K)
  int stages;                // 128-element contraction stages of the packed scales
  int tma_store;             // 1: output rows are 16-byte aligned for TMA stores
  int accumulate;            // 1: add the result into `out` (fp32 outputs, single-GPU calls)
  // Quantised output (fwd, 2-byte output types, single GPU): every 32-column
  // block of an output row is also written as MX e4m3 -- q_data, (rows,
  // out_ld) bytes -- with its e8m0 scale in q_scale, (rows, out_ld / 32)
  // row-major, quantised from the values rounded to the output type: the
  // to_mx of the output, without writing and re-reading it.  q_only: the
  // output itself is not written.
  uint8_t* q_data;
  uint8_t* q_scale;
  int q_only;
  // Transposed quantised output (same conditions; groups on the 32-row grid):
  // qt_data (out_ld, qt_rows) e4m3 holds the output's transpose quantised
  // along its rows -- to_mx(out.t()) -- with scales qt_scale (out_ld,
  // qt_rows / 32): the operand layout of the next weight-gradient pass.
  uint8_t* qt_data;
  uint8_t* qt_scale;
  long long qt_rows;
  int group_m;               // rasterisation band in row tiles (row tile fastest inside a band)
  int split_tail;            // 1: split the tiles of the last, partial round along the contraction
  int split_max;             // most pieces per split tile (0: about sqrt(stages))
  float* part_slots;         // split tiles: one fp32 128 x BN partial per CTA of the grid
  int* part_counters;        // split tiles: arrivals per (tail tile, CTA of the pair, epilogue warp), zeroed before the launch
  // Scale atoms in the blocked layout (scale_pack.cuh): [slab][stage][512 B],
  // one slab per 128 rows -- fwd A: the slabs of each group in turn, every
  // group starting a new slab; fwd B: ceil(N / 128) slabs per expert; wgrad:
  // ceil(rows / 128) slabs of each operand.  The scale writers read them
  // directly.
  const uint8_t* sfa_atoms;
  const uint8_t* sfb_atoms;
  uint32_t* status;          // error word (device memory), 0 = ok
  unsigned long long wait_ns;  // limit of every bounded wait (%globaltimer ns)
  // Expert-parallel output routing (fwd): group g's rows are stored to
  // destination group_dst[g] (an output buffer, possibly a peer GPU's) from
  // row group_dst_row[g] on.  Null group_dst: every group writes `out` at its
  // own rows.  The local destination uses the TMA store map; peers get plain
  // 16-byte stores over NVLink.
  const int32_t* group_dst;
  const int32_t* group_dst_row;
  int n_dst;
  int local_dst;
  void* out_dst[kMaxDst];
  long long out_rows_dst[kMaxDst];
  // Peer inboxes (optional): a peer's full 32-row x 64-byte output blocks go
  // to its inbox as contiguous 2 KB bulk copies, block (row / 32, byte column
  // / 64) at ((row / 32) * inbox_chunks + column / 64) * 2048, in the
  // staging buffer's 64-byte swizzle; the owner unpacks them.  NVLink moves
  // 2 KB runs at several times the rate of 64-byte row pieces.
  void* inbox_dst[kMaxDst];
  int inbox_chunks;          // 64-byte chunks per output row; 0: no inboxes
  // Streaming dispatch: the rows of group g come from source id group_src[g]
  // (a rank, or one piece of a rank's rows: ids below kMaxSrc); the producer
  // loads a tile only once that id's slot of src_flags has reached src_epoch
  // (written, after its copy, by the sender).  Null: no waits.
  const int* src_flags;
  int src_epoch;
  const int32_t* group_src;  // source id of each group's rows (null: group_dst, the rows' owner)
  // Rows of source self_src are read in place through the second A map
  // (row + self_row_base) instead of from the receive buffer; they never wait.
  int self_src;              // -1: none
  int self_row_base;
};

// Output tensor maps: [0] the output of a single-GPU call; for an
// expert-parallel call, one per destination (index = destination).
struct OutMaps {
  CUtensorMap m[kMaxDst];
};

struct Unit {
  int a_row;         // first row of the tile in the A operand
  int b_row;         // first row of the tile in the B operand
  long long out_row; // output row of tile row 0
  int out_col;       // output column of tile column 0
  int valid_rows;    // rows of the tile owned by this unit (0 .. 128 * PAIR)
  int st_begin;      // first 128-element contraction stage (global index)
  int st_count;      // number of stages (0 = the output tile is all zeros)
  int c_begin;       // contraction range [c_begin, c_end), multiples of 32
  int c_end;
  int a_sub;         // A scale slab of the tile's first 128 rows (the pair's second CTA: a_sub + 1)
  int b_tile;        // B scale slab of the tile's first 128 columns
  int b_last;        // last B scale slab of the tile's expert (fwd) or operand (wgrad)
  int dst;           // output destination (0 unless expert-parallel routing)
  int src;           // rank the rows come from (streaming dispatch)
  // a stage range of a tail tile that other CTA pairs share
  int split;         // 1: publish a partial; the last pair to arrive writes the tile
  int tail;          // index of the tile in the tail round (its arrival counter)
  int n_contrib;     // pairs contributing to the tile: p0 .. p0 + n_contrib - 1
  int p0;
  int me;            // this pair's place among the contributors
};

template <int BN, int STAGES, int PAIR, typename OutT>
struct SmemLayout {
  static constexpr int kEpiCols = 64 / sizeof(OutT);   // 64-byte staging rows
  static constexpr int kBRows = BN / PAIR;              // B rows staged by this CTA
  // A split tile's last pair sums the partials through the stage buffers,
  // idle by then: a quarter per epilogue warp, two chunk buffers of kMaxWays
  // fp32 partial chunks (32 rows x kEpiCols) each.
  static constexpr int kRedWarpBytes = (STAGES * kBM * kBK + STAGES * kBRows * kBK) / 4;
  static constexpr int kMaxWays = kRedWarpBytes / (2 * 32 * kEpiCols * 4);
  alignas(1024) uint8_t a[STAGES][kBM * kBK];
  alignas(1024) uint8_t b[STAGES][kBRows * kBK];
  alignas(1024) uint8_t epi[4][2][32 * 64];            // per epilogue warp, double buffered
  // full: the stage's A and B tiles landed (the leader's barrier counts both
  // CTAs' bytes) and every scale writer of the pair has put its scales in TMEM
  alignas(8) uint64_t full[STAGES];
  uint64_t empty[STAGES];             // stage read by its MMAs (commit to both CTAs)
  uint64_t tfull[2];
  uint64_t tempty_ov[2];    // accumulator columns shared with the other buffer drained
  uint64_t tempty_all[2];   // whole accumulator drained
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int num_units;
  int g_start[kMaxGroups];
  int g_end[kMaxGroups];
  int g_cum[kMaxGroups + 1];
  int g_cum128[kMaxGroups + 1];   // fwd: exclusive prefix of 128-row scale slabs per group
  int g_order[kMaxGroups];   // wgrad: groups by decreasing token count
  int g_expert[kMaxGroups];  // fwd: B slice of each group
  int g_dst[kMaxGroups];     // fwd, expert parallel: output destination of each group
  int g_dst_row[kMaxGroups]; //   and its first row there
  int g_src[kMaxGroups];     // fwd, streaming dispatch: source rank of each group's rows

  // a and b are one contiguous region (the split-tile reduction spans both)
  static_assert(sizeof(a) % 1024 == 0, "stage buffers must be contiguous");
};

__device__ __forceinline__ int cdiv_i(int a, int b) { return (a + b - 1) / b; }

// Group table: start/end rows (fwd) or token ranges (wgrad) per group, an
// exclusive prefix of tile rows (of `tile_m` rows each) and one of 128-row
// scale slabs.  Offsets are clamped
// into [0, R] and made monotone so that out-of-range or decreasing offsets can
// never address memory outside the operands.
template <class S>
__device__ __forceinline__ void build_group_table(S* sm, const GemmParams& p, int R, int tile_m) {
  const int lane = ptx::lane_id();
  int carry_max = 0, carry_sum = 0, carry_sum128 = 0;
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
    int t = (i < p.E) ? cdiv_i(end - start, tile_m) : 0;
    int t128 = (i < p.E) ? cdiv_i(end - start, kBM) : 0;
    int incl = t, incl128 = t128;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, incl, o);
      int u128 = __shfl_up_sync(0xffffffffu, incl128, o);
      if (lane >= o) {
        incl += u;
        incl128 += u128;
      }
    }
    if (i < p.E) {
      sm->g_start[i] = start;
      sm->g_end[i] = end;
      sm->g_cum[i] = carry_sum + incl - t;
      sm->g_cum128[i] = carry_sum128 + incl128 - t128;
    }
    carry_max = __shfl_sync(0xffffffffu, v, 31);
    carry_sum += __shfl_sync(0xffffffffu, incl, 31);
    carry_sum128 += __shfl_sync(0xffffffffu, incl128, 31);
  }
  if (lane == 0) {
    sm->g_cum[p.E] = carry_sum;
    sm->g_cum128[p.E] = carry_sum128;
  }
  // fwd: which B slice each group multiplies (clamped, so a bad index can
  // never address memory outside B)
  for (int i = lane; i < p.E; i += 32) {
    sm->g_expert[i] = p.group_expert ? min(max(__ldg(p.group_expert + i), 0), p.n_experts - 1) : i;
    if (p.group_dst) {
      sm->g_dst[i] = min(max(__ldg(p.group_dst + i), 0), p.n_dst - 1);
      sm->g_dst_row[i] = max(__ldg(p.group_dst_row + i), 0);
      sm->g_src[i] = p.group_src ? min(max(__ldg(p.group_src + i), 0), kMaxSrc - 1) : sm->g_dst[i];
    } else {
      sm->g_dst[i] = 0;
      sm->g_dst_row[i] = -1;
      sm->g_src[i] = 0;
    }
  }
}

// wgrad work per tile is proportional to the group's token count: visit the
// largest groups first so that the snake-ordered static schedule
// (unit_at) spreads big and small tiles evenly over the CTAs.
template <class S>
__device__ __forceinline__ void build_group_order(S* sm, int E) {
  const int lane = ptx::lane_id();
  for (int i = lane; i < E; i += 32) {
    const int si = sm->g_end[i] - sm->g_start[i];
    int rank = 0;
    for (int j = 0; j < E; ++j) {
      const int sj = sm->g_end[j] - sm->g_start[j];
      rank += (sj > si) || (sj == si && j < i);
    }
    sm->g_order[rank] = i;
  }
}

// k-th unit of the CTA (pair) `i` of `P`: rounds of P consecutive units,
// alternately dealt forwards and backwards, so the costliest units of every
// round do not always land on the same CTAs.
__device__ __forceinline__ int unit_at(int k, int i, int P) { return k * P + ((k & 1) ? (P - 1 - i) : i); }

template <int BN, int TILE_M, class S>
__device__ __forceinline__ Unit decode_unit(const S* sm, const GemmParams& p, int t) {
  Unit u;
  u.split = 0;
  u.dst = 0;
  u.src = 0;
  u.tail = 0;
  u.n_contrib = 1;
  u.p0 = 0;
  u.me = 0;
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
    const int row0 = sm->g_start[g] + (m - sm->g_cum[g]) * TILE_M;
    u.a_row = row0;
    const int ge = sm->g_expert[g];
    u.b_row = ge * p.N + n * BN;
    u.dst = sm->g_dst[g];
    u.src = sm->g_src[g];
    u.out_row = (sm->g_dst_row[g] >= 0) ? (long long)sm->g_dst_row[g] + (row0 - sm->g_start[g]) : row0;
    u.out_col = n * BN;
    u.valid_rows = min(TILE_M, sm->g_end[g] - row0);
    u.st_begin = 0;
    u.st_count = cdiv_i(p.K, kBK);
    u.c_begin = 0;
    u.c_end = p.K;
    u.a_sub = sm->g_cum128[g] + (m - sm->g_cum[g]) * (TILE_M / kBM);
    const int NB = cdiv_i(p.N, kBM);
    u.b_tile = ge * NB + n * (BN / kBM);
    u.b_last = ge * NB + NB - 1;
  } else {
    const int NT = cdiv_i(p.N, TILE_M);
    const int KT = cdiv_i(p.K, BN);
    const int gi = t / (NT * KT);
    const int g = sm->g_order[gi];
    // inside a group: bands of group_m row tiles (of GO_t), row tile fastest,
    // as in the forward pass
    const int r = t - gi * NT * KT;
    const int gm = p.group_m;
    const int band = r / (gm * KT);
    const int rb = r - band * gm * KT;
    const int m0 = band * gm;
    const int gsz = min(gm, NT - m0);
    const int kt = rb / gsz;
    const int nt = m0 + (rb - kt * gsz);
    const int s = sm->g_start[g], e = sm->g_end[g];
    u.a_row = nt * TILE_M;
    u.b_row = kt * BN;
    u.out_row = (long long)g * p.N + nt * TILE_M;
    u.out_col = kt * BN;
    u.valid_rows = min(TILE_M, p.N - nt * TILE_M);
    if (e > s) {
      u.st_begin = s / kBK;
      u.st_count = cdiv_i(e, kBK) - u.st_begin;
    } else {
      u.st_begin = 0;
      u.st_count = 0;
    }
    u.c_begin = s;
    u.c_end = e;
    u.a_sub = nt * (TILE_M / kBM);
    u.b_tile = kt * (BN / kBM);
    u.b_last = cdiv_i(p.K, kBM) - 1;
  }
  return u;
}

// Pieces a tail tile of C stages is split into when s pairs are free for it.
// Measured on B200 (256 x 256 pair tiles): a stage takes ~0.55 us, publishing
// a partial ~3.5 us and the last pair's reduction ~1.7 us per piece, so w
// pieces cost ~0.55 C / w + 3.5 + 1.7 w: about sqrt(C / 3) pieces, and tiles
// under 24 stages stay whole.
__device__ __forceinline__ int split_ways(const GemmParams& p, int C, int s, int max_ways) {
  if (C <= 1) return 1;
  int cap = p.split_max;
  if (cap <= 0) {
    if (C < 24) return 1;
    cap = 2;
    while ((cap + 1) * (cap + 1) * 3 <= C) ++cap;
  }
  return max(1, min(min(min(s, C), cap), max_ways));
}

// The next unit of CTA pair `pair` of `P`, identical in every role.  Whole
// tiles are dealt in snake-ordered rounds of P (units_at).  With split_tail,
// the L < P tiles of the last, partial round are instead cut along the
// contraction into pieces, one per otherwise idle pair: pair i takes piece
// i % s of tail tile i / s (s = P / L).  `k` counts the pair's rounds.
template <int BN, int TILE_M, bool kSplit, class S>
__device__ __forceinline__ bool next_unit(const S* sm, const GemmParams& p, int& k, int pair, int P, int num_units,
                                          Unit& u) {
  const int F = num_units / P;
  const int L = num_units - F * P;
  const int s = (kSplit && p.split_tail && L > 0) ? P / L : 1;
  if (s < 2 || k < F) {
    const int t = unit_at(k, pair, P);
    if (t >= num_units) return false;
    ++k;
    u = decode_unit<BN, TILE_M>(sm, p, t);
    return true;
  }
  if (k > F) return false;
  ++k;
  const int ti = pair / s, j = pair - ti * s;
  if (ti >= L) return false;
  u = decode_unit<BN, TILE_M>(sm, p, F * P + ti);
  const int C = u.st_count;
  const int ways = split_ways(p, C, s, S::kMaxWays);
  if (j >= ways) return false;
  if (ways > 1) {
    const int lo = C * j / ways, hi = C * (j + 1) / ways;
    u.st_begin += lo;
    u.st_count = hi - lo;
    u.split = 1;
    u.tail = ti;
    u.n_contrib = ways;
    u.p0 = ti * s;
    u.me = j;
  }
  return true;
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

// the two 16-bit values of a pack2 word, as floats
template <typename OutT>
__device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b);
template <>
__device__ __forceinline__ void unpack2<__nv_bfloat16>(uint32_t w, float& a, float& b) {
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xFFFF0000u);
}
template <>
__device__ __forceinline__ void unpack2<__half>(uint32_t w, float& a, float& b) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  a = f.x;
  b = f.y;
}

// One 32-column block of one output row (16 pack2 words) -> 32 e4m3 bytes at
// q and the block's e8m0 scale, with the rows-mode quantiser's arithmetic.
template <typename OutT>
__device__ __forceinline__ void quantize_block32(const uint32_t (&w)[16], uint8_t* q, uint8_t* scale) {
  float f[32];
  uint32_t amax = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) unpack2<OutT>(w[i], f[2 * i], f[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = max(amax, abs_bits(f[i]));
  const uint32_t sc = floor_scale(amax, 8);
  const float mult = __uint_as_float((254u - sc) << 23);    // 2^(127 - s)
  uint2 b[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) b[k] = e4m3x8(*reinterpret_cast<const float(*)[8]>(f + 8 * k), mult, amax);
  uint4* q4 = reinterpret_cast<uint4*>(q);
  q4[0] = make_uint4(b[0].x, b[0].y, b[1].x, b[1].y);
  q4[1] = make_uint4(b[2].x, b[2].y, b[3].x, b[3].y);
  *scale = (uint8_t)sc;
}

__device__ __forceinline__ void raise_error(const GemmParams& p, volatile int* abort, uint32_t code) {
  atomicOr(p.status, code);
  *abort = 1;
}

// Bounded wait (p.wait_ns of %globaltimer, or an abort) for source `src`'s
// rows; then orders them before this thread's TMA (async-proxy) reads.
__device__ __forceinline__ bool wait_source(const GemmParams& p, int src, volatile int* abort) {
  const int* flag = p.src_flags + src;
  const uint64_t t0 = ptx::globaltimer();
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v - p.src_epoch >= 0) break;
    if (*abort || ptx::globaltimer() - t0 > p.wait_ns) return false;
    __nanosleep(64);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// kFeat: the optional paths compiled in (kFeat* bits).  With none, the
// kernel is the plain single-GPU GEMM: measured on B200, that build of the
// same source ran the Llama4 sweep points 2-20 % faster than the one with
// every path (geomean +9 % on eight points x fwd/wgrad, the small-K points
// most), its hot loops fitting the instruction caches of the four
// sub-partitions; without the split tail, whole tiles ran another 3 % faster.
template <int BN, int STAGES, int ACC, int PAIR, typename OutT, int kFeat>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_a_self,
                        const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ OutMaps omaps,
                        const GemmParams p) {
  static_assert(BN % 128 == 0 && BN <= 256, "BN must be 128 or 256");
  static_assert(PAIR == 1 || PAIR == 2, "one CTA or a CTA pair per tile");
  static_assert(ACC == 2, "two accumulator buffers (overlapping when 2*BN does not fit)");
  constexpr bool kSplit = (kFeat & kFeatSplit) != 0;
  constexpr bool kEp = (kFeat & kFeatEp) != 0;
  constexpr bool kQuant = (kFeat & kFeatQuant) != 0;
  constexpr bool kAcc = (kFeat & kFeatAcc) != 0;
  // a scale writer waits on the empty barrier kSfSlots stages back, which must
  // be a barrier the producer has not re-armed yet
  constexpr int kSfSlots = (STAGES - 1 < kSfSlotsMax) ? STAGES - 1 : kSfSlotsMax;
  using S = SmemLayout<BN, STAGES, PAIR, OutT>;
  constexpr int kEpiCols = S::kEpiCols;
  constexpr int kChunks = BN / kEpiCols;       // epilogue chunks per accumulator
  constexpr int kTileM = kBM * PAIR;
  constexpr int kBRows = S::kBRows;
  // TMEM columns of one scale slot: the A atom (4 columns: 128 rows x 4
  // k-blocks, rows r, r+32, r+64, r+96 side by side in lane r % 32 of every
  // quarter) and BN/128 B atoms
  constexpr int kSfCols = 4 + BN / 32;
  constexpr int kSfNeed = kSfSlots * kSfCols;
  // Accumulator buffers: buffer 1 starts kOv columns before the end of buffer
  // 0 when two full buffers and the scale slots do not fit in 512 columns
  // (BN = 256).  The epilogue drains the shared columns first and releases
  // them early, so the next tile's MMAs wait for those epilogue chunks, not
  // for the whole drain.
  constexpr int kOv = (2 * BN + kSfNeed <= kTmemCols)
                          ? 0 : (2 * BN + kSfNeed - kTmemCols + kEpiCols - 1) / kEpiCols * kEpiCols;
  constexpr int kAcc1 = BN - kOv;
  constexpr int kSfCol0 = kAcc1 + BN;          // the scale slots follow the accumulators
  static_assert(kSfCol0 + kSfNeed <= kTmemCols, "tensor memory budget");
  // epilogue chunks drained first for each buffer (the shared columns)
  constexpr int kOvChunks = kOv / kEpiCols;
  // bytes one stage's tile loads deliver to the leader's full barrier (the
  // transaction count, both CTAs): e2m1 B tiles count their packed global
  // bytes, half of the 8-bit-slot smem they fill
  const uint32_t kStageBytes = PAIR * (kBM * kBK + (p.b_fmt == 5 ? kBRows * kBK / 2 : kBRows * kBK));

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  S* sm = reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort = &sm->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = (PAIR == 2) ? ptx::cluster_ctarank() : 0u;
  const bool leader = (rank == 0);
  const int unit0 = blockIdx.x / PAIR;         // pair (or CTA) index
  const int unit_stride = gridDim.x / PAIR;

  // shared::cluster address of a barrier in the pair's leader CTA
  auto leader_bar = [&](const uint64_t* bar) -> uint32_t {
    const uint32_t a = ptx::smem_u32(bar);
    return (PAIR == 2) ? ptx::mapa(a, 0) : a;
  };
  auto arrive_leader = [&](const uint64_t* bar) {
    if constexpr (PAIR == 2) ptx::mbar_arrive_cluster(leader_bar(bar));
    else ptx::mbar_arrive(ptx::smem_u32(bar));
  };
  auto wait_leader_side = [&](const uint64_t* bar, uint32_t parity) -> bool {
    if constexpr (PAIR == 2) return ptx::mbar_wait_cluster(ptx::smem_u32(bar), parity, abort, p.wait_ns);
    else return ptx::mbar_wait(ptx::smem_u32(bar), parity, abort, p.wait_ns);
  };
  // bounded wait on a barrier of this CTA
  auto wait_local = [&](const uint64_t* bar, uint32_t parity) -> bool {
    return ptx::mbar_wait(ptx::smem_u32(bar), parity, abort, p.wait_ns);
  };

  // ------------------------------------------------------------ prologue
  if (warp == kProdWarp && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // the leader's producer arms it, every CTA's tile loads complete on it,
      // and every scale-writer warp of the pair arrives on it
      ptx::mbar_init(ptx::smem_u32(&sm->full[s]), 1 + 4 * PAIR);
      ptx::mbar_init(ptx::smem_u32(&sm->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(ptx::smem_u32(&sm->tfull[a]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm->tempty_ov[a]), 4 * PAIR);    // epilogue warps of every CTA
      ptx::mbar_init(ptx::smem_u32(&sm->tempty_all[a]), 4 * PAIR);
    }
    ptx::mbar_init(ptx::smem_u32(&sm->drain), 1);
    sm->abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&omaps.m[p.local_dst]);
  }
  if (warp == kMmaWarp) {
    if constexpr (PAIR == 2) {
      ptx::tmem_alloc_pair(ptx::smem_u32(&sm->tmem_base), kTmemCols);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_u32(&sm->tmem_base), kTmemCols);
      ptx::tmem_relinquish();
    }
  }
  if (warp == 3) {
    build_group_table(sm, p, p.M, kTileM);   // fwd: rows of A; wgrad: tokens
    __syncwarp();
    if (p.mode == kWgrad) {
      build_group_order(sm, p.E);
      __syncwarp();
    }
    if (lane == 0) {
      if (p.mode == kFwd)
        sm->num_units = sm->g_cum[p.E] * cdiv_i(p.N, BN);
      else
        sm->num_units = p.E * cdiv_i(p.N, kTileM) * cdiv_i(p.K, BN);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) ptx::cluster_sync();   // peer barriers initialised before any remote arrive
  ptx::tc_fence_after();

  const uint32_t tmem_base = sm->tmem_base;
  const int num_units = sm->num_units;

  if (warp == kProdWarp) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      int k = 0;
      Unit u;
      // sources whose rows have arrived (streaming dispatch); rows read in place are always there
      uint32_t ready = (p.self_src >= 0) ? (1u << p.self_src) : 0u;
      while (ok && next_unit<BN, kTileM, kSplit>(sm, p, k, unit0, unit_stride, num_units, u)) {
        if (kEp && p.src_flags && u.st_count > 0 && !((ready >> u.src) & 1u)) {
          if (!wait_source(p, u.src, abort)) {
            raise_error(p, abort, kErrSourceWait);
            ok = false;
            break;
          }
          ready |= 1u << u.src;
        }
        for (int s = 0; s < u.st_count; ++s, ++it) {
          const int stage = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!wait_local(&sm->empty[stage], ph ^ 1u)) {
            raise_error(p, abort, kErrProducerWait);
            ok = false;
            break;
          }
          const int st = u.st_begin + s;
          const int x = st * kBK;
          if constexpr (PAIR == 2) {
            const uint32_t fb = leader_bar(&sm->full[stage]);
            if (leader) ptx::mbar_arrive_expect_tx(ptx::smem_u32(&sm->full[stage]), kStageBytes);
            if (kEp && u.src == p.self_src)
              ptx::tma_load_2d_pair(ptx::smem_u32(sm->a[stage]), &tmap_a_self, fb, x,
                                    u.a_row + p.self_row_base + kBM * (int)rank);
            else
              ptx::tma_load_2d_pair(ptx::smem_u32(sm->a[stage]), &tmap_a, fb, x, u.a_row + kBM * (int)rank);
            ptx::tma_load_2d_pair(ptx::smem_u32(sm->b[stage]), &tmap_b, fb, x, u.b_row + kBRows * (int)rank);
          } else {
            const uint32_t fb = ptx::smem_u32(&sm->full[stage]);
            ptx::mbar_arrive_expect_tx(fb, kStageBytes);
            if (kEp && u.src == p.self_src)
              ptx::tma_load_2d(ptx::smem_u32(sm->a[stage]), &tmap_a_self, fb, x, u.a_row + p.self_row_base);
            else
              ptx::tma_load_2d(ptx::smem_u32(sm->a[stage]), &tmap_a, fb, x, u.a_row);
            ptx::tma_load_2d(ptx::smem_u32(sm->b[stage]), &tmap_b, fb, x, u.b_row);
          }
        }
      }
      if (!ok || *abort) {
        // Error path: give loads already in flight 50 ms to land before the
        // CTA retires (their barrier may never complete if a peer role stopped
        // early, so this wait is bounded by time, not by the barrier).
        const uint64_t t0 = ptx::globaltimer();
        while (ptx::globaltimer() - t0 < 50000000ull) {
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      const uint32_t kIdesc = ptx::idesc_mxf8(kTileM, BN, 0, (uint32_t)p.b_fmt);
      constexpr uint32_t kAStep = (kBM * kBK) >> 4;     // descriptor start-address step per stage
      constexpr uint32_t kBStep = (kBRows * kBK) >> 4;
      const uint64_t adesc0 = ptx::kmajor_sw128_desc(ptx::smem_u32(sm->a[0]));
      const uint64_t bdesc0 = ptx::kmajor_sw128_desc(ptx::smem_u32(sm->b[0]));
      uint32_t it = 0, ai = 0;
      bool ok = true;
      int k = 0;
      Unit u;
      for (; ok && next_unit<BN, kTileM, kSplit>(sm, p, k, unit0, unit_stride, num_units, u); ++ai) {
        const int acc = ai & 1;
        const uint32_t aph = (ai >> 1) & 1u;
        // this buffer fully drained (tile ai - 2) ...
        if (!wait_leader_side(&sm->tempty_all[acc], aph ^ 1u)) {
          raise_error(p, abort, kErrAccWait);
          break;
        }
        // ... and, with overlapping buffers, the shared columns of tile ai - 1
        if (kOv > 0 && ai >= 1 && !wait_leader_side(&sm->tempty_ov[acc ^ 1], ((ai - 1) >> 1) & 1u)) {
          raise_error(p, abort, kErrAccWait);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (acc ? kAcc1 : 0);
        uint32_t accumulate = 0;
        for (int s = 0; s < u.st_count; ++s, ++it) {
          const uint32_t stage = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          const uint32_t slot = it % kSfSlots;
          // the stage's tiles (both CTAs) and its scales in TMEM (every writer warp of the pair)
          if (!wait_leader_side(&sm->full[stage], ph)) {
            raise_error(p, abort, kErrMmaWait);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sfa_t = tmem_base + kSfCol0 + slot * kSfCols;
          const uint32_t sfb_t = sfa_t + 4;
          const uint64_t adesc = adesc0 + (uint64_t)(stage * kAStep);
          const uint64_t bdesc = bdesc0 + (uint64_t)(stage * kBStep);
          const int base = (u.st_begin + s) * kBK;
          const int j0 = max(0, (u.c_begin - base) / 32);
          const int j1 = min(4, (u.c_end - base + 31) / 32);
          auto mma = [&](int j, uint32_t accum) {
            const uint32_t id = ptx::idesc_with_sf(kIdesc, j, j);
            const uint32_t fa = sfa_t | (uint32_t(j) << 30), fb = sfb_t | (uint32_t(j) << 30);
            if constexpr (PAIR == 2)
              ptx::tc_mma_mxf8_pair(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), id, fa, fb, accum);
            else
              ptx::tc_mma_mxf8(d_tmem, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), id, fa, fb, accum);
          };
          if (j0 == 0 && j1 == 4) {
#pragma unroll
            for (int j = 0; j < 4; ++j) mma(j, (j == 0) ? accumulate : 1u);
            accumulate = 1;
          } else {
            for (int j = j0; j < j1; ++j) {
              mma(j, accumulate);
              accumulate = 1;
            }
          }
          // once these MMAs complete: the stage's buffers and its scale slot are free again
          if constexpr (PAIR == 2) ptx::tc_commit_pair(ptx::smem_u32(&sm->empty[stage]), 0x3);
          else ptx::tc_commit(ptx::smem_u32(&sm->empty[stage]));
        }
        if (!ok) break;
        if constexpr (PAIR == 2) ptx::tc_commit_pair(ptx::smem_u32(&sm->tfull[acc]), 0x3);
        else ptx::tc_commit(ptx::smem_u32(&sm->tfull[acc]));
      }
      // every MMA this thread issued has retired before TMEM is released
      if constexpr (PAIR == 2) ptx::tc_commit_pair(ptx::smem_u32(&sm->drain), 0x1);
      else ptx::tc_commit(ptx::smem_u32(&sm->drain));
      volatile int never = 0;
      if (!ptx::mbar_wait(ptx::smem_u32(&sm->drain), 0, &never, p.wait_ns)) atomicOr(p.status, kErrDrain);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    // the split-tail arrival counters are zeroed by the scale-pack kernel
    // that precedes this grid (which may have launched early, see capi.cu)
    ptx::griddep_wait();
    uint32_t ai = 0;
    int buf = 0;
    int k = 0;
    Unit u;
    for (; next_unit<BN, kTileM, kSplit>(sm, p, k, unit0, unit_stride, num_units, u); ++ai) {
      const int acc = ai & 1;
      const uint32_t aph = (ai >> 1) & 1u;
      if (!wait_local(&sm->tfull[acc], aph)) {
        raise_error(p, abort, kErrEpilogueWait);
        break;
      }
      ptx::tc_fence_after();
      const int my_row0 = kBM * (int)rank + 32 * q;         // first tile row of this warp
      const int rows_here = min(max(u.valid_rows - my_row0, 0), 32);
      const bool use_tma = p.tma_store && rows_here == 32;
      const bool zero = (u.st_count == 0);
      const uint32_t t_row = tmem_base + ((uint32_t)(32 * q) << 16) + (acc ? kAcc1 : 0);
      const long long grow = u.out_row + my_row0 + lane;    // this thread's output row
      // chunk order: the columns shared with the other buffer first
      // (buffer 0: its last kOv columns, buffer 1: its first kOv columns)
      const int c_first = (acc == 0) ? (kChunks - kOvChunks) : 0;
      // chunk ci of the accumulator (in drain order) -> v, releasing the
      // buffer's shared / whole columns to the MMA warp as they are read
      auto load_chunk = [&](int ci, int c, uint32_t (&v)[kEpiCols]) {
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
        if (ci == kOvChunks - 1 || (kOvChunks == 0 && ci == 0)) {
          // shared columns read: the next tile may start its MMAs
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(&sm->tempty_ov[acc]);
        }
        if (ci == kChunks - 1) {
          // accumulator fully read: hand the buffer back to the MMA warp
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(&sm->tempty_all[acc]);
        }
      };
      // fp32 chunk c of this thread's row -> output (TMA store through the
      // staging buffer, or predicated vector stores)
      auto emit = [&](int c, const uint32_t (&v)[kEpiCols]) {
        if (rows_here == 0) return;
        const int col0 = u.out_col + c * kEpiCols;
        if (col0 >= p.out_cols) return;
        // 64 output bytes for this thread's row
        uint32_t w[16];
        if constexpr (sizeof(OutT) == 4) {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = v[i];
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack2<OutT>(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          if (kQuant && p.qt_data != nullptr) {
            // to_mx of the transposed 32 x 32 block: stage the warp's rows
            // (64-byte swizzle, as for a TMA store), then lane j reads column
            // j down the 32 rows and quantises it as one block of row col0 + j
            // of the transpose.  Needs the warp's rows on the 32-row grid.
            const long long row0 = u.out_row + my_row0;
            if (rows_here == 32 && (row0 & 31) == 0 && row0 + 32 <= p.qt_rows) {
              uint8_t* stg = sm->epi[q][buf];
              if (lane == 0) ptx::bulk_wait_read<1>();   // a TMA store may still read this buffer
              __syncwarp();
              const uint32_t stg_u = ptx::smem_u32(stg);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t chunk = (uint32_t)(j ^ ((lane >> 1) & 3));
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(stg_u + lane * 64 + chunk * 16),
                             "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                             : "memory");
              }
              __syncwarp();
              uint32_t t[16];   // column `lane`, rows 2i and 2i + 1 in word i
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                uint16_t lo, hi;
                const uint32_t off = (uint32_t)((lane >> 3) * 16 + (lane & 7) * 2);
                const int r0 = 2 * i, r1 = 2 * i + 1;
                asm volatile("ld.shared.u16 %0, [%1];" : "=h"(lo)
                             : "r"(stg_u + r0 * 64 + ((((uint32_t)lane >> 3) ^ ((r0 >> 1) & 3)) * 16) + (off & 15))
                             : "memory");
                asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hi)
                             : "r"(stg_u + r1 * 64 + ((((uint32_t)lane >> 3) ^ ((r1 >> 1) & 3)) * 16) + (off & 15))
                             : "memory");
                t[i] = (uint32_t)lo | ((uint32_t)hi << 16);
              }
              __syncwarp();   // every lane has read the block before the buffer is written again
              const long long trow = (long long)col0 + lane;
              quantize_block32<OutT>(t, p.qt_data + trow * p.qt_rows + row0, p.qt_scale + trow * (p.qt_rows / 32) + row0 / 32);
            } else if (rows_here > 0) {
              if (lane == 0) atomicOr(p.status, kErrQtRows);
            }
          }
          if (kQuant && p.q_data != nullptr) {
            // to_mx of this row's 32 output columns (host: out_cols % 32 == 0)
            if (lane < rows_here && grow < p.out_rows)
              quantize_block32<OutT>(w, p.q_data + grow * p.out_ld + col0, p.q_scale + grow * (p.out_ld / 32) + col0 / 32);
          }
          if (kQuant && p.q_only) return;
        }
        if (kEp && u.dst != p.local_dst && rows_here < 32) {
          // A peer GPU's output, rows cut by the group edge: stage the warp's
          // rows x 64 B, then store them with 4 lanes per row, so each row's
          // 64 bytes cross NVLink as one contiguous run.  Output rows are
          // 16-byte aligned (host check).  Full 32-row blocks go by TMA below.
          uint8_t* stg = sm->epi[q][buf];
          if (lane == 0) ptx::bulk_wait_read<1>();   // a TMA store may still read this buffer
          __syncwarp();
          const uint32_t stg_u = ptx::smem_u32(stg);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t chunk = (uint32_t)(j ^ ((lane >> 1) & 3));   // 64 B swizzle
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(stg_u + lane * 64 + chunk * 16),
                         "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                         : "memory");
          }
          __syncwarp();
          OutT* base = reinterpret_cast<OutT*>(p.out_dst[u.dst]);
          const long long lim = p.out_rows_dst[u.dst];
          const int ncols = min(kEpiCols, p.out_cols - col0);
          constexpr int kPer16 = 16 / (int)sizeof(OutT);
          const int j = lane & 3;
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            const int r = pp * 8 + (lane >> 2);
            const long long orow = u.out_row + my_row0 + r;
            uint4 val;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                         : "r"(stg_u + r * 64 + ((uint32_t)(j ^ ((r >> 1) & 3))) * 16)
                         : "memory");
            if (r < rows_here && orow < lim && (j + 1) * kPer16 <= ncols)
              *reinterpret_cast<uint4*>(base + orow * p.out_ld + col0 + j * kPer16) = val;
          }
          __syncwarp();
          buf ^= 1;
          return;
        }
        if (kEp && u.dst != p.local_dst && p.inbox_chunks > 0) {
          uint8_t* stg = sm->epi[q][buf];
          if (lane == 0) ptx::bulk_wait_read<1>();   // the copy that last used this buffer has read it
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
            const long long blk = ((u.out_row + my_row0) >> 5) * p.inbox_chunks + (col0 * (int)sizeof(OutT)) / 64;
            ptx::bulk_store(static_cast<uint8_t*>(p.inbox_dst[u.dst]) + blk * 2048, ptx::smem_u32(stg), 2048);
            ptx::bulk_commit();
          }
          buf ^= 1;
          return;
        }
        if (use_tma || (kEp && u.dst != p.local_dst)) {
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
            if (kAcc && p.accumulate)
              ptx::tma_reduce_add_2d(&omaps.m[u.dst], ptx::smem_u32(stg), col0, (int)(u.out_row + my_row0));
            else
              ptx::tma_store_2d(&omaps.m[u.dst], ptx::smem_u32(stg), col0, (int)(u.out_row + my_row0));
            ptx::bulk_commit();
          }
          buf ^= 1;
        } else if (lane < rows_here && grow < p.out_rows) {
          OutT* dst = reinterpret_cast<OutT*>(p.out) + grow * p.out_ld + col0;
          const int ncols = min(kEpiCols, p.out_cols - col0);
          if (kAcc && sizeof(OutT) == 4 && p.accumulate) {
            // read-add-write; every element belongs to exactly one tile
            float* d = reinterpret_cast<float*>(dst);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j < ncols) d[j] += __uint_as_float(w[j]);
          } else if (ncols == kEpiCols && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
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
      };
      if (!kSplit || !u.split) {
        int ci0 = 0;
        if constexpr (kOvChunks > 1) {
          if (!zero) {
            // the shared chunks leave TMEM together, so the next tile's MMAs
            // wait for one TMEM read, not for their conversion and stores
            const int c0 = (acc == 0) ? c_first : 0;
            uint32_t vs[kOvChunks][kEpiCols];
#pragma unroll
            for (int i = 0; i < kOvChunks; ++i) {
              if constexpr (kEpiCols == 32)
                ptx::tmem_ld_32x32b_x32(t_row + (c0 + i) * kEpiCols, reinterpret_cast<uint32_t(&)[32]>(vs[i]));
              else
                ptx::tmem_ld_32x32b_x16(t_row + (c0 + i) * kEpiCols, reinterpret_cast<uint32_t(&)[16]>(vs[i]));
            }
            ptx::tmem_wait_ld();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(&sm->tempty_ov[acc]);
#pragma unroll
            for (int i = 0; i < kOvChunks; ++i) emit(c0 + i, vs[i]);
            ci0 = kOvChunks;
          }
        }
#pragma unroll 1
        for (int ci = ci0; ci < kChunks; ++ci) {
          const int c = (acc == 0) ? (ci < kOvChunks ? c_first + ci : ci - kOvChunks) : ci;
          uint32_t v[kEpiCols];
          load_chunk(ci, c, v);
          emit(c, v);
        }
        continue;
      }
      // Split tile.  Each contributing pair publishes its fp32 partial and
      // counts its arrival; the pair that arrives last sums all partials in
      // contributor order and writes the tile, so the result does not depend
      // on timing.  A pair that finds every other partial already published
      // skips its own and adds its accumulator in its place (same order, same
      // sum).  Partial layout: per (pair, CTA, epilogue warp) a block of
      // 32 rows, float4 i of chunk c of lane l at [(c * kV + i) * 32 + l]
      // (coalesced stores, contiguous chunks for the reduction's copies).
      constexpr int kV = kEpiCols / 4;
      constexpr int kChunkF4 = kV * 32;                 // float4 per chunk of a warp block
      auto part = [&](int pair_q) -> const float4* {
        return reinterpret_cast<const float4*>(p.part_slots) +
               (long long)((pair_q * PAIR + (int)rank) * 4 + q) * (kChunks * kChunkF4) + lane;
      };
      int* const ctr = p.part_counters + (u.tail * PAIR + (int)rank) * 4 + q;
      int seen = 0;
      if (lane == 0) seen = ptx::ld_acquire_gpu(ctr);
      seen = __shfl_sync(0xffffffffu, seen, 0);
      __syncwarp();
      const bool fast = (seen == u.n_contrib - 1);
      if (!fast) {
        float4* mine = const_cast<float4*>(part(unit0));
#pragma unroll 1
        for (int ci = 0; ci < kChunks; ++ci) {
          const int c = (acc == 0) ? (ci < kOvChunks ? c_first + ci : ci - kOvChunks) : ci;
          uint32_t v[kEpiCols];
          load_chunk(ci, c, v);
#pragma unroll
          for (int i = 0; i < kV; ++i)
            __stcg(mine + c * kChunkF4 + i * 32,
                   make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                               __uint_as_float(v[4 * i + 3])));
        }
        __threadfence();
        __syncwarp();
        int arrived = 0;
        if (lane == 0) arrived = atomicAdd(ctr, 1);
        arrived = __shfl_sync(0xffffffffu, arrived, 0);
        if (arrived != u.n_contrib - 1) continue;
        __threadfence();
      }
      // Sum chunk by chunk: cp.async streams the contributors' copies of the
      // coming chunks into a ring in this warp's quarter of the (idle) stage
      // buffers, `depth` chunks deep, while the current one is added.  Each
      // lane copies and reads only its own 16-byte slots, so its own
      // wait_group orders them; one group is committed per chunk (empty ones
      // included) so that wait_group(depth - 1) always means "chunk ci landed".
      const uint32_t red = ptx::smem_u32(sm->a) + q * S::kRedWarpBytes + lane * 16;
      constexpr int kSlots = S::kRedWarpBytes / (kChunkF4 * 16);
      const int depth = min(kSlots / u.n_contrib, 12);
      auto chunk_of = [&](int ci) { return (acc == 0) ? (ci < kOvChunks ? c_first + ci : ci - kOvChunks) : ci; };
      auto slot_addr = [&](int ci, int j) {
        return red + (uint32_t)(((ci % depth) * u.n_contrib + j) * kChunkF4 * 16);
      };
      auto prefetch = [&](int ci) {
        if (ci < kChunks) {
          const int c = chunk_of(ci);
          for (int j = 0; j < u.n_contrib; ++j) {
            if (fast && j == u.me) continue;
            const float4* src = part(u.p0 + j) + c * kChunkF4;
            const uint32_t dst = slot_addr(ci, j);
#pragma unroll
            for (int i = 0; i < kV; ++i) ptx::cp_async_16(dst + i * 32 * 16, src + i * 32);
          }
        }
        ptx::cp_async_commit();
      };
      for (int ci = 0; ci < depth - 1; ++ci) prefetch(ci);
#pragma unroll 1
      for (int ci = 0; ci < kChunks; ++ci) {
        const int c = chunk_of(ci);
        uint32_t v[kEpiCols];
        if (fast) load_chunk(ci, c, v);
        prefetch(ci + depth - 1);
        ptx::cp_async_wait_group_dyn(depth - 1);
        float sum[kEpiCols];
#pragma unroll
        for (int i = 0; i < kEpiCols; ++i) sum[i] = 0.0f;
        for (int j = 0; j < u.n_contrib; ++j) {
          const uint32_t src = slot_addr(ci, j);
          if (fast && j == u.me) {
#pragma unroll
            for (int i = 0; i < kEpiCols; ++i) sum[i] += __uint_as_float(v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < kV; ++i) {
              float4 x;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                           : "r"(src + i * 32 * 16)
                           : "memory");
              sum[4 * i] += x.x; sum[4 * i + 1] += x.y; sum[4 * i + 2] += x.z; sum[4 * i + 3] += x.w;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kEpiCols; ++i) v[i] = __float_as_uint(sum[i]);
        emit(c, v);
      }
    }
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
    // expert parallel: peers read this GPU's stores after a system-scope flag
    if (kEp && p.n_dst > 1) __threadfence_system();
  } else if (warp >= kSfWarp0 && warp < kSfWarp0 + 4) {
    // ------------------------------------------------------- scale writers
    // Lane l of warp q writes TMEM lane 32q + l of the stage's scale slot:
    // row l of the A atom (4 columns) and of each B atom (4 columns each).
    // Every quarter holds the same 32 x 16-byte atom rows, the layout the
    // block-scaled MMA reads (rows r, r+32, r+64, r+96 in lane r % 32).
    //
    // Stage it's scales go to slot it % kSfSlots once the MMAs of stage
    // it - kSfSlots, the slot's last reader, have completed (that stage's
    // empty barrier).  The stage's tiles were only requested once the MMAs
    // STAGES back completed and then cross L2, so with the atoms already in
    // registers (loaded kSfRing stages earlier) the scales are in TMEM before
    // the tiles land, and the writers' arrivals do not hold the full barrier.
    // The arrival for stage it always lands in that stage's phase of full:
    // the phase before it completed before the MMAs of stage it - STAGES were
    // issued, which precedes the completion the writer waited for.
    const int q = warp - kSfWarp0;
    const uint32_t lane_base = tmem_base + ((uint32_t)(32 * q) << 16) + kSfCol0;
    constexpr int kB = BN / 128;                  // B atoms per stage
    // last A slab: the groups' slabs end at g_cum128[E] (the exact size of a
    // blocked scale tensor the caller laid out, e.g. with the quantiser)
    const int a_last = (p.mode == kFwd) ? sm->g_cum128[p.E] - 1 : cdiv_i(p.N, kBM) - 1;
    // load cursor over the (unit, stage) sequence every role walks
    int lk = 0, ls = 0;
    Unit lu;
    bool lhas = false;
    // this lane's 16 bytes of the unit's first A and B atoms (per-unit slab
    // clamps and address arithmetic stay out of the per-stage path): stage
    // ls of the unit is 512 bytes further per stage, [ls * 32]
    const uint4* pa = nullptr;
    const uint4* pb[kB];
    auto advance = [&]() -> bool {
      while (true) {
        if (lhas && ls + 1 < lu.st_count) {
          ++ls;
          return true;
        }
        if (!next_unit<BN, kTileM, kSplit>(sm, p, lk, unit0, unit_stride, num_units, lu)) return false;
        lhas = true;
        ls = -1;
        const int sa = min(lu.a_sub + (int)rank, a_last);
        pa = reinterpret_cast<const uint4*>(p.sfa_atoms + ((long long)sa * p.stages + lu.st_begin) * 512) + lane;
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const int sb = min(lu.b_tile + b, lu.b_last);
          pb[b] = reinterpret_cast<const uint4*>(p.sfb_atoms + ((long long)sb * p.stages + lu.st_begin) * 512) + lane;
        }
      }
    };
    bool ok = true;
    // sources whose atoms may be read (streaming dispatch: a sender packs its
    // rows' atoms before it raises its flag); rows read in place are always there
    uint32_t ready = (p.self_src >= 0) ? (1u << p.self_src) : 0u;
    auto load = [&](uint4 (&r)[3]) {
      // a unit's rows come from one source: check it at the unit's first
      // stage only (checking every stage measured 20-25 % slower GEMMs)
      if (kEp && ls == 0 && p.src_flags && !((ready >> lu.src) & 1u)) {
        int got = 1;
        if (lane == 0) {
          got = wait_source(p, lu.src, abort) ? 1 : 0;
          if (!got) raise_error(p, abort, kErrSourceWait);
        }
        __syncwarp();
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          return;
        }
        int f;   // every lane's own acquire of the raised flag
        asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(f) : "l"(p.src_flags + lu.src) : "memory");
        ready |= 1u << lu.src;
      }
      // slabs past a group's or an expert's rows hold other rows' scales (or
      // are clamped to the last slab): they only feed rows that are never stored
      r[0] = __ldg(pa + ls * 32);
#pragma unroll
      for (int b = 0; b < kB; ++b) r[1 + b] = __ldg(pb[b] + ls * 32);
    };
    // the atoms are written by the scale-pack kernel that precedes this grid
    ptx::griddep_wait();
    uint4 ring[kSfRing][3];
    int loaded = 0;
#pragma unroll
    for (int r = 0; r < kSfRing; ++r) {
      if (ok && advance()) {
        load(ring[r]);
        ++loaded;
      }
    }
    uint32_t it = 0;
    bool done = false;
    while (!done) {
#pragma unroll
      for (int r = 0; r < kSfRing; ++r) {   // stage it sits in ring[it % kSfRing] == ring[r]
        if (!ok || (int)it >= loaded) {
          done = true;
          break;
        }
        if (it >= (uint32_t)kSfSlots) {
          // the slot's last reader, stage it - kSfSlots, has completed
          const uint32_t j = it - kSfSlots;
          if (!wait_local(&sm->empty[j % STAGES], (j / STAGES) & 1u)) {
            raise_error(p, abort, kErrScaleWait);
            ok = false;
            done = true;
            break;
          }
        }
        const uint32_t taddr = lane_base + (it % kSfSlots) * kSfCols;
        ptx::tmem_st_32x32b_x4(taddr, reinterpret_cast<const uint32_t(&)[4]>(ring[r][0]));
#pragma unroll
        for (int b = 0; b < kB; ++b)
          ptx::tmem_st_32x32b_x4(taddr + 4 + 4 * b, reinterpret_cast<const uint32_t(&)[4]>(ring[r][1 + b]));
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&sm->full[it % STAGES]);
        ++it;
        if (ok && advance()) {
          load(ring[r]);
          ++loaded;
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) ptx::cluster_sync();   // the peer no longer touches this CTA's barriers or smem
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    if constexpr (PAIR == 2) ptx::tmem_dealloc_pair(tmem_base, kTmemCols);
    else ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace mxgg
