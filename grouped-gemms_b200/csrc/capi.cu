// C ABI of the mxgg library (see include/mxgg.h): argument validation,
// TMA descriptor construction and kernel launches.  Host code never
// synchronises (except mxgg_device_status) and never allocates.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mxgg.h"
#include "gemm_launch.cuh"
#include "grouped_gemm.cuh"
#include "quantize.cuh"
#include "scale_pack.cuh"
#include "moe.cuh"
#include "peer.cuh"
#include "tile_map.cuh"

namespace mxgg {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define MXGG_CUDA_TRY(expr)                                                                   \
  do {                                                                                        \
    cudaError_t e_ = (expr);                                                                  \
    if (e_ != cudaSuccess) return fail(MXGG_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// device-side error word raised by bounded waits
__device__ uint32_t g_status_word;

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool init = false;
  int num_sms = 0;
  uint32_t* status = nullptr;   // device address of g_status_word
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// Tile and schedule choice of one call: the process defaults
// (mxgg_set_tile_config / mxgg_set_schedule, read under g_mu) overridden by
// the non-zero fields of the call's own mxgg_gemm_config.
struct GemmCfg {
  int tile_m = 0;
  int tile_n = 0;
  int group_m = 0;
  int schedule = MXGG_SCHED_DEFAULT;
  int split_max = 0;
  int scale_layout = MXGG_SCALE_ROW_MAJOR;   // per call only (it describes the caller's tensors)
};
GemmCfg g_default_cfg;   // guarded by g_mu
// Limit of every bounded device-side wait (mbarriers, peers' flags, the
// cross-GPU barrier), guarded by g_mu.
constexpr unsigned long long kDefaultWaitNs = 1000000000ull;   // 1 s
unsigned long long g_wait_ns = kDefaultWaitNs;

unsigned long long wait_limit_ns() {
  std::lock_guard<std::mutex> lk(g_mu);
  return g_wait_ns;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
using WriteValueFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
WriteValueFn g_write_value = nullptr;

int get_device_state(DeviceState** out) {
  int dev = 0;
  MXGG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(MXGG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    int major = 0, minor = 0;
    MXGG_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MXGG_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      return fail(MXGG_ERR_UNSUPPORTED, "mxgg kernels are built for sm_100a; device %d is sm_%d%d", dev, major,
                  minor);
    MXGG_CUDA_TRY(cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, dev));
    void* p = nullptr;
    MXGG_CUDA_TRY(cudaGetSymbolAddress(&p, g_status_word));
    st.status = static_cast<uint32_t*>(p);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      MXGG_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
      if (q != cudaDriverEntryPointSuccess || !fn)
        return fail(MXGG_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    if (!g_write_value) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      MXGG_CUDA_TRY(cudaGetDriverEntryPoint("cuStreamWriteValue32", &fn, cudaEnableDefault, &q));
      if (q == cudaDriverEntryPointSuccess && fn) g_write_value = reinterpret_cast<WriteValueFn>(fn);
    }
    st.init = true;
  }
  *out = &st;
  return MXGG_OK;
}

// 2-D tensor map over a row-major (rows, cols) matrix.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esize, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swz) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MXGG_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu stride=%llu box=%ux%u",
                (int)r, (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)row_stride_elems,
                box_rows, box_cols);
  return MXGG_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int out_esize(int out_dtype) { return out_dtype == MXGG_DTYPE_F32 ? 4 : 2; }

CUtensorMapDataType out_tmap_dtype(int out_dtype) {
  switch (out_dtype) {
    case MXGG_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case MXGG_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

// Workspace of one GEMM call: [A atoms | B atoms | split-tail partials |
// arrival counters], each part 1 KiB aligned.  The atoms (the blocked scale
// layout, scale_pack.cuh) do not depend on the tile shape; the partials do,
// so a size query takes the larger tile width.
struct WsPlan {
  long long a_slabs, b_slabs, stages, a_bytes, b_bytes;
  long long part_bytes, counter_bytes;   // split tail: one fp32 partial tile per CTA, arrival counters
  long long total;                       // with the split-tail scratch
  long long base;                        // without it
};


// fwd: E groups (segments) over n_experts slices of B; wgrad: n_experts unused
WsPlan plan_workspace(int mode, int64_t M, int64_t N, int64_t K, int64_t E, int64_t n_experts, int tile_m,
                      int tile_n) {
  WsPlan w{};
  const int64_t C = mode == kFwd ? K : M;
  w.stages = (C + kBK - 1) / kBK;
  (void)tile_m;
  if (mode == kFwd) {
    // sum over groups of ceil(rows_g / 128) <= ceil(M / 128) + E - 1
    w.a_slabs = (M + kBM - 1) / kBM + (E - 1);
    w.b_slabs = n_experts * ((N + kBM - 1) / kBM);
  } else {
    w.a_slabs = (N + kBM - 1) / kBM;
    w.b_slabs = (K + kBM - 1) / kBM;
  }
  w.a_bytes = (w.a_slabs * w.stages * 512 + 1023) / 1024 * 1024;
  w.b_bytes = (w.b_slabs * w.stages * 512 + 1023) / 1024 * 1024;
  // one fp32 128 x tile_n partial per CTA; one counter per (tail tile, CTA
  // of the pair, epilogue warp), fewer tail tiles than pairs
  w.part_bytes = (long long)kMaxGridCtas * kBM * tile_n * 4;
  w.counter_bytes = ((long long)kMaxGridCtas * 4 * 4 + 1023) / 1024 * 1024;
  w.base = w.a_bytes + w.b_bytes;
  w.total = w.base + w.part_bytes + w.counter_bytes;
  return w;
}

int64_t workspace_upper_bound(int mode, int64_t M, int64_t N, int64_t K, int64_t E, int64_t n_experts,
                              bool with_split = true) {
  int64_t best = 0;
  for (int tm : {128, 256})
    for (int tn : {128, 256}) {
      const WsPlan w = plan_workspace(mode, M, N, K, E, n_experts, tm, tn);
      best = std::max<int64_t>(best, with_split ? w.total : w.base);
    }
  return best;
}

struct TileChoice {
  int tile_m;   // 128: one CTA per tile; 256: a CTA pair per tile
  int tile_n;   // 128 or 256
};

// Default tiles: a CTA pair per 256 x 256 tile with raster bands of 16 row
// tiles (best on 101 of the 108 Llama4 sweep points against one CTA per
// 128 x 256 tile, measured in one run); single-CTA tiles prefer bands of 2.
TileChoice pick_tiles(int64_t n_extent, const GemmCfg& cfg) {
  TileChoice c;
  c.tile_m = (cfg.tile_m == 128 || cfg.tile_m == 256) ? cfg.tile_m : 256;
  c.tile_n = (cfg.tile_n == 128 || cfg.tile_n == 256) ? cfg.tile_n : (n_extent >= 256 ? 256 : 128);
  return c;
}

int pick_group_m(const TileChoice& c, const GemmCfg& cfg) {
  if (cfg.group_m > 0) return cfg.group_m;
  return c.tile_m == 128 ? 2 : 16;
}

int check_cfg_fields(int tile_m, int tile_n, int group_m, int schedule, int split_max, const char* what) {
  if (tile_m != 0 && tile_m != 128 && tile_m != 256)
    return fail(MXGG_ERR_INVALID, "%s: tile_m must be 0, 128 or 256 (got %d)", what, tile_m);
  if (tile_n != 0 && tile_n != 128 && tile_n != 256)
    return fail(MXGG_ERR_INVALID, "%s: tile_n must be 0, 128 or 256 (got %d)", what, tile_n);
  if (group_m < 0) return fail(MXGG_ERR_INVALID, "%s: group_m must be >= 0 (got %d)", what, group_m);
  if (schedule != MXGG_SCHED_DEFAULT && schedule != MXGG_SCHED_TILES && schedule != MXGG_SCHED_SPLIT_TAIL)
    return fail(MXGG_ERR_INVALID, "%s: unknown schedule %d", what, schedule);
  if (split_max < 0 || split_max == 1 || split_max > 64)
    return fail(MXGG_ERR_INVALID, "%s: split_max must be 0 (automatic) or 2..64 (got %d)", what, split_max);
  return MXGG_OK;
}

// The call's configuration: a snapshot of the process defaults taken under
// the lock (so a concurrent mxgg_set_* never tears it), with the non-zero
// fields of `user` (may be null) on top.
int resolve_cfg(const mxgg_gemm_config* user, GemmCfg* out, const char* what) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    *out = g_default_cfg;
  }
  if (!user) return MXGG_OK;
  if (user->reserved[0] || user->reserved[1])
    return fail(MXGG_ERR_INVALID, "%s: mxgg_gemm_config.reserved must be zero", what);
  if (user->scale_layout != MXGG_SCALE_ROW_MAJOR && user->scale_layout != MXGG_SCALE_BLOCKED)
    return fail(MXGG_ERR_INVALID, "%s: unknown scale_layout %d", what, user->scale_layout);
  out->scale_layout = user->scale_layout;
  if (int rc = check_cfg_fields(user->tile_m, user->tile_n, user->group_m, user->schedule, user->split_max, what))
    return rc;
  if (user->tile_m) out->tile_m = user->tile_m;
  if (user->tile_n) out->tile_n = user->tile_n;
  if (user->group_m) out->group_m = user->group_m;
  if (user->schedule != MXGG_SCHED_DEFAULT) out->schedule = user->schedule;
  if (user->split_max) out->split_max = user->split_max;
  return MXGG_OK;
}

// Expert-parallel output routing of a forward call (see GemmParams).
struct EpRoute {
  const int32_t* group_dst = nullptr;
  const int32_t* group_dst_row = nullptr;
  int n_dst = 0;
  int local_dst = 0;
  void* out_dst[kMaxDst] = {};
  int64_t rows_dst[kMaxDst] = {};
  void* inbox_dst[kMaxDst] = {};   // all null: peers' rows are stored in place
  const void* a_atoms = nullptr;   // A scale atoms packed by the senders (null: pack here)
  const int32_t* src_flags = nullptr;
  int32_t src_epoch = 0;
  const int32_t* group_src = nullptr;
  const void* a_self = nullptr;    // rows of source self_src, read in place
  int64_t a_self_rows = 0;
  int32_t self_src = -1;
  int64_t self_row_base = 0;
};

// Quantised forward output (see GemmParams::q_data).
struct QuantOut {
  void* data = nullptr;     // (M, N) e4m3 (or null)
  void* scales = nullptr;   // (M, N / 32) e8m0, row-major
  void* tdata = nullptr;    // (N, M) e4m3: the transpose, quantised along M (or null)
  void* tscales = nullptr;  // (N, M / 32) e8m0, row-major
  bool only = false;        // no high-precision output
};

// split_ok = 0: the caller's scratch only needs the packed scales and the
// tail of the schedule is dealt as whole tiles.
// Forward groups may be segments that share B slices: group g multiplies
// B[group_expert[g]] (null: B[g], n_experts == E).
int run_gemm(int mode, const void* a, const void* b, const void* a_scale, const void* b_scale,
             const int32_t* offs, int64_t M, int64_t N, int64_t K, int64_t E, void* out, int out_dtype,
             void* workspace, int64_t workspace_bytes, void* stream_v, bool split_ok = true,
             const int32_t* group_expert = nullptr, int64_t n_experts = -1,
             const char* what = nullptr, const EpRoute* route = nullptr, int b_format = MXGG_FMT_E4M3,
             bool accumulate = false, const QuantOut* quant = nullptr, const mxgg_gemm_config* user_cfg = nullptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (!what) what = mode == kFwd ? "mxgg_grouped_mm" : "mxgg_wgrad";
  GemmCfg cfg;
  if (int rc = resolve_cfg(user_cfg, &cfg, what)) return rc;
  if (n_experts < 0) n_experts = E;
  if (out_dtype != MXGG_DTYPE_BF16 && out_dtype != MXGG_DTYPE_F16 && out_dtype != MXGG_DTYPE_F32)
    return fail(MXGG_ERR_INVALID, "%s: unknown out_dtype %d", what, out_dtype);
  if (M < 0 || N < 0 || K < 0 || E < 1)
    return fail(MXGG_ERR_INVALID, "%s: bad sizes M=%lld N=%lld K=%lld E=%lld", what, (long long)M, (long long)N,
                (long long)K, (long long)E);
  if (E > kMaxGroups) return fail(MXGG_ERR_UNSUPPORTED, "%s: E=%lld exceeds %d groups", what, (long long)E, kMaxGroups);
  if (n_experts < 1) return fail(MXGG_ERR_INVALID, "%s: n_experts=%lld", what, (long long)n_experts);
  if (b_format != MXGG_FMT_E4M3 && b_format != MXGG_FMT_E2M1)
    return fail(MXGG_ERR_INVALID, "%s: unknown B format %d", what, b_format);
  const bool b_fp4 = b_format == MXGG_FMT_E2M1;
  if (accumulate && (out_dtype != MXGG_DTYPE_F32 || route))
    return fail(MXGG_ERR_UNSUPPORTED, "%s: accumulating into the output needs an fp32 output on one GPU", what);
  if (b_fp4 && (mode != kFwd || K % 128 != 0 || !aligned(b, 32)))
    return fail(MXGG_ERR_UNSUPPORTED, "%s: e2m1 weights need the forward pass, K %% 128 == 0 and a 32-byte "
                "aligned B", what);
  // contraction length: fwd K, wgrad tokens M
  const int64_t C = mode == kFwd ? K : M;
  const int64_t rows_a = mode == kFwd ? M : N;
  const int64_t rows_b = mode == kFwd ? n_experts * N : K;
  const int64_t out_cols = mode == kFwd ? N : K;
  int64_t out_rows = mode == kFwd ? M : E * N;
  if (C % 32 != 0)
    return fail(MXGG_ERR_INVALID, "%s: contraction length %lld must be a multiple of 32", what, (long long)C);
  const int es_out = out_esize(out_dtype);
  if (quant) {
    bool local_rows = true;   // an expert-parallel call may quantise only rows that stay on this GPU
    if (route)
      for (int i = 0; i < route->n_dst && i < kMaxDst; ++i)
        if (i != route->local_dst && route->rows_dst[i] != 0) local_rows = false;
    if (mode != kFwd || !local_rows || accumulate || es_out != 2 || out_cols % 32 != 0)
      return fail(MXGG_ERR_UNSUPPORTED, "%s: a quantised output needs the forward pass with every row stored on "
                  "this GPU, a bf16 or f16 output type and N %% 32 == 0 (N = %lld)", what, (long long)out_cols);
    if (out_rows > 0 && out_cols > 0) {
      if (!quant->data && !quant->tdata)
        return fail(MXGG_ERR_INVALID, "%s: no quantised output buffer", what);
      if (quant->data && (!quant->scales || !aligned(quant->data, 16)))
        return fail(MXGG_ERR_INVALID, "%s: the quantised output needs a 16-byte aligned data buffer and a scale "
                    "buffer", what);
      if (quant->tdata && (!quant->tscales || !aligned(quant->tdata, 16) || out_rows % 32 != 0))
        return fail(MXGG_ERR_INVALID, "%s: the transposed quantised output needs M %% 32 == 0 (M = %lld), a "
                    "16-byte aligned data buffer and a scale buffer", what, (long long)out_rows);
    }
  }
  const bool out_written = !(quant && quant->only);
  if (route) {
    if (mode != kFwd || route->n_dst < 1 || route->n_dst > kMaxDst || route->local_dst < 0 ||
        route->local_dst >= route->n_dst || !route->group_dst || !route->group_dst_row)
      return fail(MXGG_ERR_INVALID, "%s: bad expert-parallel routing (n_dst %d, local %d)", what, route->n_dst,
                  route->local_dst);
    if (C == 0 || (out_cols * es_out) % 16 != 0)
      return fail(MXGG_ERR_UNSUPPORTED, "%s: expert-parallel outputs need K > 0 and 16-byte output rows", what);
    for (int i = 0; i < route->n_dst; ++i) {
      if (i == route->local_dst && !out_written && !route->out_dst[i]) continue;   // quantised rows only
      if (route->rows_dst[i] < 0 || (route->rows_dst[i] > 0 && (!route->out_dst[i] || !aligned(route->out_dst[i], 16))))
        return fail(MXGG_ERR_INVALID, "%s: destination %d needs a 16-byte aligned output", what, i);
    }
    out = route->out_dst[route->local_dst];
    out_rows = route->rows_dst[route->local_dst];
    if (M == 0 || out_cols == 0) return MXGG_OK;
  } else {
    if (out_rows == 0 || out_cols == 0) return MXGG_OK;
    if (!out && out_written) return fail(MXGG_ERR_INVALID, "%s: null output", what);
    if (!out_written) out = nullptr;
  }
  const int64_t lim = (int64_t)1 << 31;
  if (rows_a >= lim || rows_b >= lim || out_rows >= lim || C >= lim || out_cols >= lim)
    return fail(MXGG_ERR_UNSUPPORTED, "%s: extents beyond 2^31", what);
  if (C == 0) {
    // empty contraction: every product is the zero accumulator (the
    // reference's loops run zero times and store zeros, backward.py:67,
    // forward.py:207-212); accumulating zeros changes nothing
    if (!accumulate && out)
      MXGG_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)(out_rows * out_cols * out_esize(out_dtype)), stream));
    if (quant) {
      // zero blocks quantise to zero codes with scale 0 (FLT_MIN's exponent - 8 clamps to 0)
      if (quant->data) {
        MXGG_CUDA_TRY(cudaMemsetAsync(quant->data, 0, (size_t)(out_rows * out_cols), stream));
        MXGG_CUDA_TRY(cudaMemsetAsync(quant->scales, 0, (size_t)(out_rows * (out_cols / 32)), stream));
      }
      if (quant->tdata) {
        MXGG_CUDA_TRY(cudaMemsetAsync(quant->tdata, 0, (size_t)(out_rows * out_cols), stream));
        MXGG_CUDA_TRY(cudaMemsetAsync(quant->tscales, 0, (size_t)((out_rows / 32) * out_cols), stream));
      }
    }
    return MXGG_OK;
  }
  if (!a || !b || !a_scale || !b_scale || !offs) return fail(MXGG_ERR_INVALID, "%s: null input pointer", what);
  if (!aligned(a, 16) || !aligned(b, 16))
    return fail(MXGG_ERR_INVALID, "%s: e4m3 operands must be 16-byte aligned", what);

  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;

  const TileChoice tc = pick_tiles(out_cols, cfg);
  const int bn = tc.tile_n;
  const int pair = tc.tile_m / kBM;
  const WsPlan ws = plan_workspace(mode, M, N, K, E, n_experts, tc.tile_m, bn);
  const long long need = split_ok ? ws.total : ws.base;
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(MXGG_ERR_INVALID, "%s: workspace of %lld bytes (256-byte aligned) required, got %lld at %p", what,
                need, (long long)workspace_bytes, workspace);
  uint8_t* ws_a = static_cast<uint8_t*>(workspace);
  uint8_t* ws_b = ws_a + ws.a_bytes;
  float* part_slots = reinterpret_cast<float*>(ws_b + ws.b_bytes);
  int* part_counters = reinterpret_cast<int*>(ws_b + ws.b_bytes + ws.part_bytes);
  // A tile splits only if it has enough stages (the kernel's split_ways: at
  // least 2 with a split_max, else at least 24): when none can, the split
  // machinery -- and the zeroing of its counters -- stays off.
  const long long max_stages = mode == kFwd ? ws.stages : ws.stages + 1;   // a group's tokens may straddle one more
  const bool split_tail = split_ok && cfg.schedule == MXGG_SCHED_SPLIT_TAIL &&
                          (cfg.split_max > 0 ? max_stages >= 2 : max_stages >= 24);
  const bool blocked = cfg.scale_layout == MXGG_SCALE_BLOCKED;
  if (blocked && (route || !aligned(a_scale, 16) || !aligned(b_scale, 16)))
    return fail(MXGG_ERR_INVALID, "%s: blocked scales must be 16-byte aligned (and are not taken by the "
                "expert-parallel call)", what);

  if (blocked) {
    // the scales are laid out already; only the split-tail counters need zeros
    if (split_tail) MXGG_CUDA_TRY(cudaMemsetAsync(part_counters, 0, (size_t)ws.counter_bytes, stream));
  } else {
    // 1) pack the row-major scales into the blocked atoms the GEMM reads
    PackParams pp{};
    pp.mode = mode;
    pp.E = (int)E;
    pp.stages = (int)ws.stages;
    pp.offs = offs;
    pp.sfa = static_cast<const uint8_t*>(a_scale);
    pp.sfb = static_cast<const uint8_t*>(b_scale);
    pp.rows_a = (int)rows_a;
    pp.rows_b = (int)rows_b;
    pp.sf_ld = C / 32;
    const int64_t ld = C / 32;
    if (ld % 16 == 0 && aligned(a_scale, 16) && aligned(b_scale, 16)) pp.vec = 4;
    else if (ld % 4 == 0 && aligned(a_scale, 4) && aligned(b_scale, 4)) pp.vec = 1;
    else pp.vec = 0;
    // A atoms the senders packed already: pack only B here
    pp.a_slabs = (route && route->a_atoms) ? 0 : (int)ws.a_slabs;
    pp.b_slabs = (int)ws.b_slabs;
    pp.b_height = (int)(mode == kFwd ? N : K);
    pp.a_out = ws_a;
    pp.b_out = ws_b;
    if (split_tail) {
      pp.zero = part_counters;
      pp.zero_count = ws.counter_bytes / 4;
    }
    const long long chunks = (ws.stages + 3) / 4;
    const long long warps = ((long long)pp.a_slabs + pp.b_slabs) * chunks;
    const long long blocks = std::max(1LL, std::min<long long>((warps + 7) / 8, (long long)st->num_sms * 8));
    pack_scales_kernel<<<(unsigned)blocks, 256, 0, stream>>>(pp);
    MXGG_CUDA_TRY(cudaGetLastError());
  }

  GemmParams p{};
  p.mode = mode;
  p.E = (int)E;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.rows_a = (int)rows_a;
  p.rows_b = (int)rows_b;
  p.contraction = (int)C;
  p.offs = offs;
  p.group_expert = mode == kFwd ? group_expert : nullptr;
  p.n_experts = (int)n_experts;
  p.b_fmt = b_fp4 ? 5 : 0;
  p.stages = (int)ws.stages;
  p.out = out;
  p.out_ld = out_cols;
  p.out_rows = out_rows;
  p.out_cols = (int)out_cols;
  const int es = out_esize(out_dtype);
  p.tma_store = out != nullptr && out_rows > 0 && aligned(out, 16) && ((out_cols * es) % 16 == 0);
  if (quant) {
    p.q_data = static_cast<uint8_t*>(quant->data);
    p.q_scale = static_cast<uint8_t*>(quant->scales);
    p.qt_data = static_cast<uint8_t*>(quant->tdata);
    p.qt_scale = static_cast<uint8_t*>(quant->tscales);
    p.qt_rows = out_rows;
    p.q_only = out_written ? 0 : 1;
  }
  if (route) {
    p.group_dst = route->group_dst;
    p.group_dst_row = route->group_dst_row;
    p.n_dst = route->n_dst;
    p.local_dst = route->local_dst;
    bool inbox = (out_cols * es) % 64 == 0;
    for (int i = 0; i < route->n_dst; ++i) {
      p.out_dst[i] = route->out_dst[i];
      p.out_rows_dst[i] = route->rows_dst[i];
      p.inbox_dst[i] = route->inbox_dst[i];
      if (i != route->local_dst && route->rows_dst[i] > 0 && (!route->inbox_dst[i] || !aligned(route->inbox_dst[i], 16)))
        inbox = false;
    }
    p.inbox_chunks = inbox ? (int)((out_cols * es) / 64) : 0;
    p.src_flags = route->src_flags;
    p.src_epoch = route->src_epoch;
    p.group_src = route->group_src;
    p.self_src = route->a_self ? route->self_src : -1;
    p.self_row_base = (int)route->self_row_base;
  } else {
    p.n_dst = 1;
    p.local_dst = 0;
    p.out_dst[0] = out;
    p.out_rows_dst[0] = out_rows;
    p.self_src = -1;
  }
  p.group_m = pick_group_m(tc, cfg);
  p.accumulate = accumulate ? 1 : 0;
  p.split_tail = split_tail ? 1 : 0;
  p.split_max = cfg.split_max;
  p.part_slots = part_slots;
  p.part_counters = part_counters;
  p.status = st->status;
  p.wait_ns = wait_limit_ns();

  Maps maps;
  if (int rc = make_tmap_2d(&maps.a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)rows_a, (uint64_t)C, (uint64_t)C,
                            kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (route && route->a_self && route->a_self_rows > 0) {
    if (!aligned(route->a_self, 16)) return fail(MXGG_ERR_INVALID, "%s: in-place rows must be 16-byte aligned", what);
    if (int rc = make_tmap_2d(&maps.a_self, route->a_self, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1,
                              (uint64_t)route->a_self_rows, (uint64_t)C, (uint64_t)C, kBK, kBM,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    maps.a_self = maps.a;
  }
  // e2m1 weights: packed two per byte in HBM; TMA's 16U4_ALIGN16B type
  // spreads every 16 values (8 bytes) over a 16-byte slot, the 8-bit
  // container layout kind::mxf8f6f4 reads, so the smem tile and its
  // descriptors are the same as for e4m3.
  if (int rc = b_fp4 ? make_tmap_2d(&maps.b, b, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 1, (uint64_t)rows_b,
                                    (uint64_t)C, (uint64_t)(C / 2), kBK, (uint32_t)(bn / pair),
                                    CU_TENSOR_MAP_SWIZZLE_128B)
                     : make_tmap_2d(&maps.b, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)rows_b, (uint64_t)C,
                                    (uint64_t)C, kBK, (uint32_t)(bn / pair), CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  // the scale writers read the packed atoms directly; every slab index they
  // form is clamped inside the a_slabs x stages and b_slabs x stages atoms
  if (blocked) {
    p.sfa_atoms = static_cast<const uint8_t*>(a_scale);
    p.sfb_atoms = static_cast<const uint8_t*>(b_scale);
  } else {
    p.sfa_atoms = static_cast<const uint8_t*>((route && route->a_atoms) ? route->a_atoms : ws_a);
    p.sfb_atoms = ws_b;
  }
  std::memset(&maps.out, 0, sizeof(maps.out));
  if (route) {
    // one map per destination with rows (the peers' outputs take TMA stores too)
    for (int i = 0; i < route->n_dst; ++i) {
      if (route->rows_dst[i] <= 0 || !route->out_dst[i]) continue;
      if (int rc = make_tmap_2d(&maps.out.m[i], route->out_dst[i], out_tmap_dtype(out_dtype), es,
                                (uint64_t)route->rows_dst[i], (uint64_t)out_cols, (uint64_t)out_cols, 64 / es, 32,
                                CU_TENSOR_MAP_SWIZZLE_64B))
        return rc;
    }
  } else if (p.tma_store) {
    if (int rc = make_tmap_2d(&maps.out.m[0], out, out_tmap_dtype(out_dtype), es, (uint64_t)out_rows,
                              (uint64_t)out_cols, (uint64_t)out_cols, 64 / es, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
  }

  long long max_units;
  const int tile_m = tc.tile_m;
  if (mode == kFwd) {
    const long long mt_ub = (M + tile_m - 1) / tile_m + (E - 1);
    max_units = mt_ub * ((N + bn - 1) / bn);
  } else {
    max_units = E * ((N + tile_m - 1) / tile_m) * ((K + bn - 1) / bn);
  }
  // the kernel build with the optional paths this call uses (the plain
  // build, whole tiles, for the reference's calls)
  int feat = 0;
  if (split_tail) feat |= kFeatSplit;
  if (route) feat |= kFeatEp;
  if (quant) feat |= kFeatQuant;
  if (accumulate) feat |= kFeatAcc;
  int dev = 0;
  MXGG_CUDA_TRY(cudaGetDevice(&dev));
  const GemmLaunch l{dev, st->num_sms, &maps, &p, max_units, out_dtype, bn, pair, stream};
  cudaError_t e;
  if (feat == 0) e = launch_gemm_plain(l);
  else if (feat == kFeatSplit) e = launch_gemm_split(l);
  else if (feat == kFeatEp) e = launch_gemm_ep(l);
  else e = launch_gemm_full(l);
  if (e != cudaSuccess) return fail(MXGG_ERR_CUDA, "%s: GEMM launch: %s", what, cudaGetErrorString(e));
  return MXGG_OK;
}

// Scratch of mxgg_grouped_mm_noalloc: a fixed array in device memory that
// every GPU which loads this library holds until the process exits.  Host
// code cannot use the name `g_noalloc_scratch` as an address (on the host it
// is only a stand-in object); the device address comes from
// cudaGetSymbolAddress, once per device, with that device current.
constexpr int64_t kNoAllocScratchBytes = 32ll << 20;   // 32 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_ptr[kMaxDevices] = {};

}  // namespace
}  // namespace mxgg

using namespace mxgg;

extern "C" {

int64_t mxgg_grouped_mm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t E) {
  if (M < 0 || N < 0 || K < 0 || E < 1) return -1;
  return workspace_upper_bound(kFwd, M, N, K, E, E);
}

int64_t mxgg_wgrad_workspace_size(int64_t N, int64_t K, int64_t M, int64_t E) {
  if (M < 0 || N < 0 || K < 0 || E < 1) return -1;
  return workspace_upper_bound(kWgrad, M, N, K, E, E);
}

int mxgg_grouped_mm(const void* a, const void* b, const void* a_scale, const void* b_scale,
                    const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E, void* out,
                    int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  return run_gemm(kFwd, a, b, a_scale, b_scale, group_end_offsets, M, N, K, E, out, out_dtype, workspace,
                  workspace_bytes, stream);
}

int mxgg_grouped_mm_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                        const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E, void* out,
                        int out_dtype, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  return run_gemm(kFwd, a, b, a_scale, b_scale, group_end_offsets, M, N, K, E, out, out_dtype, workspace,
                  workspace_bytes, stream, true, nullptr, -1, "mxgg_grouped_mm_cfg", nullptr, MXGG_FMT_E4M3, false,
                  nullptr, config);
}

int64_t mxgg_grouped_mm_segments_workspace_size(int64_t M, int64_t N, int64_t K, int64_t n_segments,
                                                int64_t n_experts) {
  if (M < 0 || N < 0 || K < 0 || n_segments < 1 || n_experts < 1) return -1;
  return workspace_upper_bound(kFwd, M, N, K, n_segments, n_experts);
}

int mxgg_grouped_mm_segments(const void* a, const void* b, const void* a_scale, const void* b_scale,
                             const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                             int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out,
                             int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!segment_expert && n_segments > 0) return fail(MXGG_ERR_INVALID, "mxgg_grouped_mm_segments: null segment_expert");
  return run_gemm(kFwd, a, b, a_scale, b_scale, segment_end_offsets, M, N, K, n_segments, out, out_dtype, workspace,
                  workspace_bytes, stream, true, segment_expert, n_experts, "mxgg_grouped_mm_segments", nullptr,
                  b_format);
}

int mxgg_grouped_mm_segments_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                 const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M,
                                 int64_t N, int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format,
                                 void* out, int out_dtype, const mxgg_gemm_config* config, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  if (!segment_expert && n_segments > 0)
    return fail(MXGG_ERR_INVALID, "mxgg_grouped_mm_segments_cfg: null segment_expert");
  return run_gemm(kFwd, a, b, a_scale, b_scale, segment_end_offsets, M, N, K, n_segments, out, out_dtype, workspace,
                  workspace_bytes, stream, true, segment_expert, n_experts, "mxgg_grouped_mm_segments_cfg", nullptr,
                  b_format, false, nullptr, config);
}

int mxgg_grouped_mm_mx_cfg(const void* a, const void* b, const void* a_scale, const void* b_scale,
                           const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                           int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out,
                           int out_dtype, void* q_out, void* q_scales, void* qt_out, void* qt_scales,
                           const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes, void* stream) {
  QuantOut q;
  q.data = q_out;
  q.scales = q_scales;
  q.tdata = qt_out;
  q.tscales = qt_scales;
  q.only = out == nullptr;
  return run_gemm(kFwd, a, b, a_scale, b_scale, segment_end_offsets, M, N, K, n_segments, out, out_dtype, workspace,
                  workspace_bytes, stream, true, segment_expert, segment_expert ? n_experts : n_segments,
                  "mxgg_grouped_mm_mx_cfg", nullptr, b_format, false, &q, config);
}

int mxgg_grouped_mm_mx(const void* a, const void* b, const void* a_scale, const void* b_scale,
                       const int32_t* segment_end_offsets, const int32_t* segment_expert, int64_t M, int64_t N,
                       int64_t K, int64_t n_segments, int64_t n_experts, int32_t b_format, void* out, int out_dtype,
                       void* q_out, void* q_scales, void* qt_out, void* qt_scales, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  QuantOut q;
  q.data = q_out;
  q.scales = q_scales;
  q.tdata = qt_out;
  q.tscales = qt_scales;
  q.only = out == nullptr;
  return run_gemm(kFwd, a, b, a_scale, b_scale, segment_end_offsets, M, N, K, n_segments, out, out_dtype, workspace,
                  workspace_bytes, stream, true, segment_expert, segment_expert ? n_experts : n_segments,
                  "mxgg_grouped_mm_mx", nullptr, b_format, false, &q);
}

int mxgg_grouped_mm_noalloc(const void* a, const void* b, const void* a_scale, const void* b_scale,
                            const int32_t* group_end_offsets, int64_t M, int64_t N, int64_t K, int64_t E,
                            void* out, int out_dtype, void* stream) {
  bool split_ok = true;
  if (M >= 0 && N >= 0 && K >= 0 && E >= 1) {
    const int64_t need = workspace_upper_bound(kFwd, M, N, K, E, E, false);
    // the split tail needs its partial tiles too; without room for them the
    // last round is dealt as whole tiles
    split_ok = workspace_upper_bound(kFwd, M, N, K, E, E, true) <= kNoAllocScratchBytes;
    if (need > kNoAllocScratchBytes)
      return fail(MXGG_ERR_UNSUPPORTED,
                  "mxgg_grouped_mm_noalloc: this problem needs %lld bytes of scratch, more than the %lld-byte "
                  "static array; call mxgg_grouped_mm with a workspace instead",
                  (long long)need, (long long)kNoAllocScratchBytes);
  }
  int dev = 0;
  MXGG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(MXGG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_noalloc_ptr[dev]) {
      // first call on this device: resolve the array's device address
      void* p = nullptr;
      MXGG_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      g_noalloc_ptr[dev] = p;
    }
    ws = g_noalloc_ptr[dev];
  }
  return run_gemm(kFwd, a, b, a_scale, b_scale, group_end_offsets, M, N, K, E, out, out_dtype, ws,
                  kNoAllocScratchBytes, stream, split_ok);
}

int mxgg_wgrad(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
               const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, void* out,
               int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  return run_gemm(kWgrad, go_t, ia_t, go_scale, ia_scale, group_end_offsets, M, N, K, E, out, out_dtype, workspace,
                  workspace_bytes, stream);
}

int mxgg_wgrad_cfg(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                   const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, void* out,
                   int out_dtype, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                   void* stream) {
  return run_gemm(kWgrad, go_t, ia_t, go_scale, ia_scale, group_end_offsets, M, N, K, E, out, out_dtype, workspace,
                  workspace_bytes, stream, true, nullptr, -1, "mxgg_wgrad_cfg", nullptr, MXGG_FMT_E4M3, false,
                  nullptr, config);
}

int mxgg_quantize_mx_gather(const void* x, int x_dtype, int64_t in_rows, const int32_t* row_index, int64_t n_rows,
                            int64_t cols, void* q, void* scales, void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (in_rows < 0 || n_rows < 0 || cols < 0) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_gather: negative size");
  if (n_rows == 0 || cols == 0) return MXGG_OK;
  if (!x || !row_index || !q || !scales) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_gather: null pointer");
  if (x_dtype != MXGG_DTYPE_BF16 && x_dtype != MXGG_DTYPE_F16 && x_dtype != MXGG_DTYPE_F32)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_gather: unknown x_dtype %d", x_dtype);
  if (cols % 32 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_gather: cols=%lld not a multiple of 32", (long long)cols);
  if (!aligned(x, 16) || !aligned(q, 8))
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_gather: x must be 16-byte and q 8-byte aligned");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long work = n_rows * cols / 8;
  const long long blocks = std::max(1LL, std::min<long long>((work + 255) / 256, (long long)st->num_sms * 16));
  uint8_t* qq = static_cast<uint8_t*>(q);
  uint8_t* ss = static_cast<uint8_t*>(scales);
  switch (x_dtype) {
    case MXGG_DTYPE_BF16:
      quantize_rows_gather_e4m3<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), in_rows, row_index, n_rows, cols, qq, ss);
      break;
    case MXGG_DTYPE_F16:
      quantize_rows_gather_e4m3<__half><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const __half*>(x),
                                                                              in_rows, row_index, n_rows, cols, qq, ss);
      break;
    default:
      quantize_rows_gather_e4m3<float><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const float*>(x), in_rows,
                                                                             row_index, n_rows, cols, qq, ss);
  }
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_quantize_mx_fp4(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales,
                         int scale_layout, void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (rows < 0 || cols < 0) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: negative size");
  if (rows == 0 || cols == 0) return MXGG_OK;
  if (!x || !q || !scales) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: null pointer");
  if (x_dtype != MXGG_DTYPE_BF16 && x_dtype != MXGG_DTYPE_F16 && x_dtype != MXGG_DTYPE_F32)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: unknown x_dtype %d", x_dtype);
  if (scale_layout != MXGG_SCALE_ROW_MAJOR && scale_layout != MXGG_SCALE_BLOCKED)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: unknown scale layout %d", scale_layout);
  if (cols % 32 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: cols=%lld not a multiple of 32", (long long)cols);
  if (!aligned(x, 16) || !aligned(q, 4))
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx_fp4: x must be 16-byte and q 4-byte aligned");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const int nthreads = 256;
  const long long work = rows * cols / 8;
  const long long blocks =
      std::max(1LL, std::min<long long>((work + nthreads - 1) / nthreads, (long long)st->num_sms * 8));
  uint8_t* qq = static_cast<uint8_t*>(q);
  uint8_t* ss = static_cast<uint8_t*>(scales);
  switch (x_dtype) {
    case MXGG_DTYPE_BF16:
      quantize_rows_e4m3<__nv_bfloat16, true><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), rows, cols, qq, ss, scale_layout, ScaleSegs{});
      break;
    case MXGG_DTYPE_F16:
      quantize_rows_e4m3<__half, true><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const __half*>(x), rows, cols, qq, ss, scale_layout, ScaleSegs{});
      break;
    default:
      quantize_rows_e4m3<float, true><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const float*>(x), rows, cols, qq, ss, scale_layout, ScaleSegs{});
  }
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_wgrad_accumulate(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                          const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E, float* out,
                          void* workspace, int64_t workspace_bytes, void* stream) {
  return run_gemm(kWgrad, go_t, ia_t, go_scale, ia_scale, group_end_offsets, M, N, K, E, out, MXGG_DTYPE_F32,
                  workspace, workspace_bytes, stream, true, nullptr, -1, "mxgg_wgrad_accumulate", nullptr,
                  MXGG_FMT_E4M3, true);
}

int mxgg_wgrad_accumulate_cfg(const void* go_t, const void* go_scale, const void* ia_t, const void* ia_scale,
                              const int32_t* group_end_offsets, int64_t N, int64_t K, int64_t M, int64_t E,
                              float* out, const mxgg_gemm_config* config, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  return run_gemm(kWgrad, go_t, ia_t, go_scale, ia_scale, group_end_offsets, M, N, K, E, out, MXGG_DTYPE_F32,
                  workspace, workspace_bytes, stream, true, nullptr, -1, "mxgg_wgrad_accumulate_cfg", nullptr,
                  MXGG_FMT_E4M3, true, nullptr, config);
}

int mxgg_quantize_mx(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales, int mode,
                     int scale_layout, void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (rows < 0 || cols < 0) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: negative size");
  if (rows == 0 || cols == 0) return MXGG_OK;
  if (!x || !q || !scales) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: null pointer");
  if (x_dtype != MXGG_DTYPE_BF16 && x_dtype != MXGG_DTYPE_F16 && x_dtype != MXGG_DTYPE_F32)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: unknown x_dtype %d", x_dtype);
  if (scale_layout != MXGG_SCALE_ROW_MAJOR && scale_layout != MXGG_SCALE_BLOCKED)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: unknown scale layout %d", scale_layout);
  if (!aligned(x, 16) || !aligned(q, 8))
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: x must be 16-byte and q 8-byte aligned");
  if (mode != MXGG_QUANT_ROWS && mode != MXGG_QUANT_COLS)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: unknown mode %d", mode);
  if (mode == MXGG_QUANT_ROWS && cols % 32 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: cols=%lld not a multiple of 32", (long long)cols);
  if (mode == MXGG_QUANT_COLS && rows % 32 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: rows=%lld not a multiple of 32", (long long)rows);
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const int nthreads = 256;
  if (mode == MXGG_QUANT_ROWS) {
    if (cols % 32 != 0) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: cols=%lld not a multiple of 32", (long long)cols);
    const long long work = rows * cols / 8;
    const long long blocks = std::max(1LL, std::min<long long>((work + nthreads - 1) / nthreads, (long long)st->num_sms * 8));
    switch (x_dtype) {
      case MXGG_DTYPE_BF16:
        quantize_rows_e4m3<__nv_bfloat16><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout,
            ScaleSegs{});
        break;
      case MXGG_DTYPE_F16:
        quantize_rows_e4m3<__half><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const __half*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout,
            ScaleSegs{});
        break;
      default:
        quantize_rows_e4m3<float><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const float*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout,
            ScaleSegs{});
    }
  } else if (mode == MXGG_QUANT_COLS) {
    if (rows % 32 != 0) return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: rows=%lld not a multiple of 32", (long long)rows);
    if (cols % 8 != 0) return fail(MXGG_ERR_UNSUPPORTED, "mxgg_quantize_mx: column mode needs cols %% 8 == 0");
    const long long tiles = (rows / 32) * ((cols + 63) / 64);
    const long long blocks = std::max(1LL, std::min<long long>(tiles, (long long)st->num_sms * 8));
    switch (x_dtype) {
      case MXGG_DTYPE_BF16:
        quantize_cols_e4m3<__nv_bfloat16><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout);
        break;
      case MXGG_DTYPE_F16:
        quantize_cols_e4m3<__half><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const __half*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout);
        break;
      default:
        quantize_cols_e4m3<float><<<(unsigned)blocks, nthreads, 0, stream>>>(
            static_cast<const float*>(x), rows, cols, static_cast<uint8_t*>(q), static_cast<uint8_t*>(scales), scale_layout);
    }
  } else {
    return fail(MXGG_ERR_INVALID, "mxgg_quantize_mx: unknown mode %d", mode);
  }
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int64_t mxgg_blocked_scale_bytes(int64_t rows, int64_t contraction, int64_t n_segments) {
  if (rows < 0 || contraction < 0 || n_segments < 1) return -1;
  const int64_t slabs = (rows + 127) / 128 + (n_segments - 1);
  return slabs * ((contraction + 127) / 128) * 512;
}

int mxgg_quantize_mx_blocked(const void* x, int x_dtype, int64_t rows, int64_t cols, void* q, void* scales,
                             const int32_t* segment_end_offsets, int64_t n_segments, int64_t segment_rows,
                             void* stream_v) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const char* what = "mxgg_quantize_mx_blocked";
  if (rows < 0 || cols < 0) return fail(MXGG_ERR_INVALID, "%s: negative size", what);
  if (n_segments < 1 || n_segments > kMaxScaleSegments)
    return fail(MXGG_ERR_INVALID, "%s: n_segments=%lld outside 1..%d", what, (long long)n_segments,
                kMaxScaleSegments);
  if (!segment_end_offsets && segment_rows < 1)
    return fail(MXGG_ERR_INVALID, "%s: uniform segments need segment_rows >= 1", what);
  if (rows == 0 || cols == 0) return MXGG_OK;
  if (!x || !q || !scales) return fail(MXGG_ERR_INVALID, "%s: null pointer", what);
  if (x_dtype != MXGG_DTYPE_BF16 && x_dtype != MXGG_DTYPE_F16 && x_dtype != MXGG_DTYPE_F32)
    return fail(MXGG_ERR_INVALID, "%s: unknown x_dtype %d", what, x_dtype);
  if (cols % 32 != 0) return fail(MXGG_ERR_INVALID, "%s: cols=%lld not a multiple of 32", what, (long long)cols);
  if (!aligned(x, 16) || !aligned(q, 8))
    return fail(MXGG_ERR_INVALID, "%s: x must be 16-byte and q 8-byte aligned", what);
  if (rows >= ((int64_t)1 << 31)) return fail(MXGG_ERR_UNSUPPORTED, "%s: rows beyond 2^31", what);
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const ScaleSegs segs{segment_end_offsets, (int)n_segments, segment_end_offsets ? 0 : (long long)segment_rows};
  const int nthreads = 256;
  const long long work = rows * cols / 8;
  const long long blocks = std::max(1LL, std::min<long long>((work + nthreads - 1) / nthreads, (long long)st->num_sms * 8));
  uint8_t* qq = static_cast<uint8_t*>(q);
  uint8_t* ss = static_cast<uint8_t*>(scales);
  switch (x_dtype) {
    case MXGG_DTYPE_BF16:
      quantize_rows_e4m3<__nv_bfloat16><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), rows, cols, qq, ss, kScaleBlockedSeg, segs);
      break;
    case MXGG_DTYPE_F16:
      quantize_rows_e4m3<__half><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const __half*>(x), rows, cols, qq, ss, kScaleBlockedSeg, segs);
      break;
    default:
      quantize_rows_e4m3<float><<<(unsigned)blocks, nthreads, 0, stream>>>(
          static_cast<const float*>(x), rows, cols, qq, ss, kScaleBlockedSeg, segs);
  }
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_grouped_mm_ep(const void* a, const void* b, const void* a_scale, const void* b_scale,
                       const int32_t* segment_end_offsets, const int32_t* segment_expert, const int32_t* segment_dst,
                       const int32_t* segment_dst_row, int64_t M, int64_t N, int64_t K, int64_t n_segments,
                       int64_t n_experts, int32_t b_format, void* const* dst_out, const int64_t* dst_rows,
                       void* const* dst_inbox, int32_t n_dst, int32_t local_dst, const void* a_atoms,
                       const int32_t* src_flags, int32_t src_epoch, const int32_t* segment_src,
                       const void* a_self, int64_t a_self_rows, int32_t self_src, int64_t self_row_base,
                       void* q_out, void* q_scales, int out_dtype, void* workspace, int64_t workspace_bytes,
                       void* stream) {
  if (!segment_expert || !dst_out || !dst_rows)
    return fail(MXGG_ERR_INVALID, "mxgg_grouped_mm_ep: null segment or destination table");
  if (n_dst < 1 || n_dst > kMaxDst)
    return fail(MXGG_ERR_UNSUPPORTED, "mxgg_grouped_mm_ep: %d destinations (1..%d)", (int)n_dst, kMaxDst);
  EpRoute r;
  r.group_dst = segment_dst;
  r.group_dst_row = segment_dst_row;
  r.n_dst = n_dst;
  r.local_dst = local_dst;
  for (int i = 0; i < n_dst; ++i) {
    r.out_dst[i] = dst_out[i];
    r.rows_dst[i] = dst_rows[i];
    r.inbox_dst[i] = dst_inbox ? dst_inbox[i] : nullptr;
  }
  if (a_atoms && !aligned(a_atoms, 256)) return fail(MXGG_ERR_INVALID, "mxgg_grouped_mm_ep: a_atoms not 256-byte aligned");
  r.a_atoms = a_atoms;
  r.src_flags = src_flags;
  r.src_epoch = src_epoch;
  r.group_src = segment_src;
  if (a_self && (self_src < 0 || self_src >= n_dst || self_row_base < 0))
    return fail(MXGG_ERR_INVALID, "mxgg_grouped_mm_ep: bad in-place source %d", (int)self_src);
  r.a_self = a_self;
  r.a_self_rows = a_self_rows;
  r.self_src = self_src;
  r.self_row_base = self_row_base;
  QuantOut q;
  if (q_out) {
    q.data = q_out;
    q.scales = q_scales;
    q.only = local_dst >= 0 && local_dst < n_dst && dst_out[local_dst] == nullptr;
  }
  return run_gemm(kFwd, a, b, a_scale, b_scale, segment_end_offsets, M, N, K, n_segments, nullptr, out_dtype,
                  workspace, workspace_bytes, stream, true, segment_expert, n_experts, "mxgg_grouped_mm_ep", &r,
                  b_format, false, q_out ? &q : nullptr);
}

int32_t mxgg_query_tile_m(void) {
  GemmCfg cfg;
  resolve_cfg(nullptr, &cfg, "mxgg_query_tile_m");
  return pick_tiles(256, cfg).tile_m;
}

int64_t mxgg_ep_atom_bytes(int64_t M, int64_t K, int64_t n_segments) {
  if (M < 0 || K < 0 || n_segments < 1) return -1;
  return plan_workspace(kFwd, M, 128, K, n_segments, 1, 256, 256).a_bytes;
}

// PackParams of one forward-A atom pack (mxgg_pack_a_atoms); returns the warps it needs.
static long long a_atom_pack_params(const void* a_scale, const int32_t* segment_end_offsets, int64_t rows, int64_t K,
                                    int64_t n_segments, void* out, PackParams* pp) {
  *pp = PackParams{};
  pp->mode = kFwd;
  pp->E = (int)n_segments;
  pp->stages = (int)((K + kBK - 1) / kBK);
  pp->offs = segment_end_offsets;
  pp->sfa = static_cast<const uint8_t*>(a_scale);
  pp->sfb = static_cast<const uint8_t*>(a_scale);
  pp->rows_a = (int)rows;
  pp->rows_b = 1;
  pp->sf_ld = K / 32;
  const int64_t ld = K / 32;
  pp->vec = (ld % 16 == 0 && aligned(a_scale, 16)) ? 4 : ((ld % 4 == 0 && aligned(a_scale, 4)) ? 1 : 0);
  pp->a_slabs = (int)((rows + kBM - 1) / kBM + (n_segments - 1));
  pp->b_slabs = 0;
  pp->b_height = 1;
  pp->a_out = static_cast<uint8_t*>(out);
  pp->b_out = nullptr;
  return (long long)pp->a_slabs * ((pp->stages + 3) / 4);
}

int mxgg_pack_a_atoms(const void* a_scale, const int32_t* segment_end_offsets, int64_t rows, int64_t K,
                      int64_t n_segments, void* out, void* stream) {
  if (rows < 0 || K <= 0 || K % 32 != 0 || n_segments < 1 || n_segments > kMaxGroups)
    return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms: bad sizes (rows %lld, K %lld, segments %lld)",
                (long long)rows, (long long)K, (long long)n_segments);
  if (rows == 0) return MXGG_OK;
  if (!a_scale || !segment_end_offsets || !out) return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms: null pointer");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  PackParams pp;
  const long long warps = a_atom_pack_params(a_scale, segment_end_offsets, rows, K, n_segments, out, &pp);
  const long long blocks = std::max(1LL, std::min<long long>((warps + 7) / 8, (long long)st->num_sms * 8));
  pack_scales_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(pp);
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_pack_a_atoms_multi(const void* a_scale, int64_t K, int32_t n_dst, const int64_t* first_row,
                            const int64_t* rows, const int32_t* const* segment_end_offsets,
                            const int64_t* n_segments, void* const* out, void* stream) {
  if (n_dst < 0 || n_dst > kMaxDst || K <= 0 || K % 32 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms_multi: bad sizes (n_dst %d, K %lld)", (int)n_dst, (long long)K);
  if (n_dst == 0) return MXGG_OK;
  if (!a_scale || !first_row || !rows || !segment_end_offsets || !n_segments || !out)
    return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms_multi: null pointer");
  PackMulti m{};
  int n = 0;
  long long warps = 0;
  for (int i = 0; i < n_dst; ++i) {
    if (rows[i] < 0 || first_row[i] < 0 || n_segments[i] < 1 || n_segments[i] > kMaxGroups)
      return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms_multi: bad sizes of pack %d (rows %lld, segments %lld)", i,
                  (long long)rows[i], (long long)n_segments[i]);
    if (rows[i] == 0) continue;
    if (!segment_end_offsets[i] || !out[i])
      return fail(MXGG_ERR_INVALID, "mxgg_pack_a_atoms_multi: null pointer in pack %d", i);
    const void* src = static_cast<const uint8_t*>(a_scale) + first_row[i] * (K / 32);
    warps = std::max(warps, a_atom_pack_params(src, segment_end_offsets[i], rows[i], K, n_segments[i], out[i], &m.p[n]));
    ++n;
  }
  if (n == 0) return MXGG_OK;
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long blocks = std::max(1LL, std::min<long long>((warps + 7) / 8, (long long)st->num_sms * 8 / n + 1));
  pack_scales_multi_kernel<<<dim3((unsigned)blocks, (unsigned)n), 256, 0, static_cast<cudaStream_t>(stream)>>>(m);
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

// A stream memory operation, not a kernel: it needs no SM, so it cannot be
// held back by a GEMM that fills the GPU while waiting for the very flags
// such signals raise on its peers.
int mxgg_peer_signal(void* slot, int32_t epoch, void* stream) {
  if (!slot || !aligned(slot, 4)) return fail(MXGG_ERR_INVALID, "mxgg_peer_signal: bad slot");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  if (!g_write_value) return fail(MXGG_ERR_UNSUPPORTED, "mxgg_peer_signal: cuStreamWriteValue32 is not available");
  CUresult r = g_write_value(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(slot), (cuuint32_t)epoch,
                             CU_STREAM_WRITE_VALUE_DEFAULT);
  if (r != CUDA_SUCCESS) return fail(MXGG_ERR_CUDA, "mxgg_peer_signal: cuStreamWriteValue32 failed (%d)", (int)r);
  return MXGG_OK;
}

int mxgg_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  if (bytes <= 0 || !ptr || !handle) return fail(MXGG_ERR_INVALID, "mxgg_ipc_alloc: bad arguments");
  void* p = nullptr;
  MXGG_CUDA_TRY(cudaMalloc(&p, (size_t)bytes));
  if (cudaError_t e = cudaMemset(p, 0, (size_t)bytes)) {
    cudaFree(p);
    return fail(MXGG_ERR_CUDA, "mxgg_ipc_alloc: %s", cudaGetErrorString(e));
  }
  cudaIpcMemHandle_t h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h, p)) {
    cudaFree(p);
    return fail(MXGG_ERR_CUDA, "mxgg_ipc_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MXGG_OK;
}

int mxgg_ipc_free(void* ptr) {
  MXGG_CUDA_TRY(cudaFree(ptr));
  return MXGG_OK;
}

int mxgg_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(MXGG_ERR_INVALID, "mxgg_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MXGG_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MXGG_OK;
}

int mxgg_ipc_close(void* ptr) {
  MXGG_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return MXGG_OK;
}

int mxgg_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0) return fail(MXGG_ERR_INVALID, "mxgg_copy_async: negative size");
  if (bytes == 0) return MXGG_OK;
  MXGG_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return MXGG_OK;
}

int mxgg_peer_barrier(void* const* flags, int32_t world, int32_t rank, int32_t epoch, void* stream) {
  if (!flags || world < 1 || world > kMaxDst || rank < 0 || rank >= world)
    return fail(MXGG_ERR_INVALID, "mxgg_peer_barrier: bad arguments (world %d, rank %d)", (int)world, (int)rank);
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  PeerFlags f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return fail(MXGG_ERR_INVALID, "mxgg_peer_barrier: null flag array of rank %d", i);
    f.flags[i] = static_cast<int*>(flags[i]);
  }
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, world, rank, epoch, st->status,
                                                                      wait_limit_ns());
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_replica_sum(void* const* bufs, int32_t n, int32_t me, int64_t elems, int dtype, void* stream) {
  if (!bufs || n < 1 || n > kMaxDst || me < 0 || me >= n || elems < 0)
    return fail(MXGG_ERR_INVALID, "mxgg_replica_sum: bad arguments (n %d, me %d, elems %lld)", (int)n, (int)me,
                (long long)elems);
  const int es = dtype == MXGG_DTYPE_F32 ? 4 : (dtype == MXGG_DTYPE_BF16 || dtype == MXGG_DTYPE_F16) ? 2 : 0;
  if (es == 0) return fail(MXGG_ERR_INVALID, "mxgg_replica_sum: unknown dtype %d", dtype);
  if ((elems * es) % 16 != 0)
    return fail(MXGG_ERR_UNSUPPORTED, "mxgg_replica_sum: %lld bytes is not a multiple of 16", (long long)(elems * es));
  ReplicaBufs b{};
  for (int i = 0; i < n; ++i) {
    if (!bufs[i] || !aligned(bufs[i], 16))
      return fail(MXGG_ERR_INVALID, "mxgg_replica_sum: null or unaligned buffer of replica %d", i);
    b.p[i] = static_cast<uint8_t*>(bufs[i]);
  }
  if (n == 1 || elems == 0) return MXGG_OK;
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long chunks = elems * es / 16;
  const long long lo = chunks * me / n, hi = chunks * (me + 1) / n;
  if (hi <= lo) return MXGG_OK;
  const unsigned blocks = (unsigned)std::max(1LL, std::min<long long>((hi - lo + 255) / 256, (long long)st->num_sms * 8));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == MXGG_DTYPE_F32) launch_replica_sum<float>(b, n, lo, hi, blocks, s);
  else if (dtype == MXGG_DTYPE_BF16) launch_replica_sum<__nv_bfloat16>(b, n, lo, hi, blocks, s);
  else launch_replica_sum<__half>(b, n, lo, hi, blocks, s);
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_inbox_unpack(const void* inbox, void* out, const int32_t* row_blocks, int64_t n_row_blocks,
                      int64_t row_bytes, void* stream) {
  if (n_row_blocks < 0 || row_bytes <= 0 || row_bytes % 64 != 0)
    return fail(MXGG_ERR_INVALID, "mxgg_inbox_unpack: row_bytes %lld must be a positive multiple of 64",
                (long long)row_bytes);
  if (n_row_blocks == 0) return MXGG_OK;
  if (!inbox || !out || !row_blocks || !aligned(inbox, 16) || !aligned(out, 16))
    return fail(MXGG_ERR_INVALID, "mxgg_inbox_unpack: null or unaligned pointer");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long warps = n_row_blocks * (row_bytes / 64);
  const long long blocks = std::max(1LL, std::min<long long>((warps + 7) / 8, (long long)st->num_sms * 8));
  inbox_unpack_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(inbox), static_cast<uint8_t*>(out), row_blocks, (int)n_row_blocks,
      (int)(row_bytes / 64), (long long)row_bytes);
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_combine_topk(const void* y, int64_t y_rows, const int64_t* pos, const float* weights, int64_t tokens,
                      int64_t N, int32_t k, void* out, void* stream) {
  if (tokens < 0 || N < 0 || k < 1 || y_rows < 0) return fail(MXGG_ERR_INVALID, "mxgg_combine_topk: bad sizes");
  if (tokens == 0 || N == 0) return MXGG_OK;
  if (N % 8 != 0) return fail(MXGG_ERR_UNSUPPORTED, "mxgg_combine_topk: N %% 8 != 0");
  if (!y || !pos || !weights || !out || !aligned(y, 16) || !aligned(out, 16))
    return fail(MXGG_ERR_INVALID, "mxgg_combine_topk: null or unaligned pointer");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long blocks = std::max(1LL, std::min<long long>((tokens + 7) / 8, (long long)st->num_sms * 16));
  combine_topk_bf16<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), pos, weights, y_rows, (int)tokens, (int)N, (int)k,
      static_cast<__nv_bfloat16*>(out));
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_build_tile_map(const int32_t* offs, int64_t E, int64_t M, int32_t block_m, int32_t* out, void* stream_v) {
  if (E < 1 || M < 0 || block_m < 1 || !offs || !out)
    return fail(MXGG_ERR_INVALID, "mxgg_build_tile_map: bad arguments");
  if (E > (1 << 16)) return fail(MXGG_ERR_UNSUPPORTED, "mxgg_build_tile_map: E beyond 65536");
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  const long long grid_m_ub = (M + block_m - 1) / block_m + (E - 1);
  const long long n = 2 * E + 1 + grid_m_ub;
  tile_map_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream_v)>>>(
      offs, (int)E, (int)block_m, (int)grid_m_ub, out);
  MXGG_CUDA_TRY(cudaGetLastError());
  return MXGG_OK;
}

int mxgg_set_tile_config(int32_t tile_m, int32_t tile_n, int32_t group_m) {
  if (int rc = check_cfg_fields(tile_m, tile_n, group_m, MXGG_SCHED_DEFAULT, 0, "mxgg_set_tile_config")) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  g_default_cfg.tile_m = tile_m;
  g_default_cfg.tile_n = tile_n;
  g_default_cfg.group_m = group_m;
  return MXGG_OK;
}

int mxgg_set_schedule(int32_t schedule, int32_t split_max) {
  if (int rc = check_cfg_fields(0, 0, 0, schedule, split_max, "mxgg_set_schedule")) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  g_default_cfg.schedule = schedule;
  g_default_cfg.split_max = split_max;
  return MXGG_OK;
}

int mxgg_set_wait_limit(int64_t ns) {
  if (ns < 0 || (ns > 0 && ns < 1000000) || ns > 60000000000ll)
    return fail(MXGG_ERR_INVALID, "mxgg_set_wait_limit: %lld ns is outside 1 ms .. 60 s (0 restores 1 s)",
                (long long)ns);
  std::lock_guard<std::mutex> lk(g_mu);
  g_wait_ns = ns == 0 ? kDefaultWaitNs : (unsigned long long)ns;
  return MXGG_OK;
}

int64_t mxgg_wait_limit(void) { return (int64_t)wait_limit_ns(); }

int mxgg_device_status(uint32_t* status_out, int clear, void* stream_v) {
  DeviceState* st = nullptr;
  if (int rc = get_device_state(&st)) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  uint32_t v = 0;
  MXGG_CUDA_TRY(cudaMemcpyAsync(&v, st->status, sizeof(v), cudaMemcpyDeviceToHost, stream));
  MXGG_CUDA_TRY(cudaStreamSynchronize(stream));
  if (clear) {
    MXGG_CUDA_TRY(cudaMemsetAsync(st->status, 0, sizeof(uint32_t), stream));
    MXGG_CUDA_TRY(cudaStreamSynchronize(stream));
  }
  if (status_out) *status_out = v;
  return MXGG_OK;
}

const char* mxgg_last_error(void) { return g_last_error.c_str(); }

int32_t mxgg_version(void) { return 1; }

#ifndef MXGG_BUILD_ID
#define MXGG_BUILD_ID "unversioned"
#endif
const char* mxgg_build_id(void) { return MXGG_BUILD_ID; }

}  // extern "C"
