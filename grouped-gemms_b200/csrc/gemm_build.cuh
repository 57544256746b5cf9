// The templated launcher of one grouped-GEMM build, included by the
// gemm_build_*.cu translation units only.
#pragma once

#include <algorithm>

#include "../../include/mxgg.h"
#include "gemm_launch.cuh"

namespace mxgg {
// Internal to each build's translation unit: a function-local static of a
// template with external linkage would be one object shared by every copy of
// the library loaded in the process (a unique symbol), so a second copy
// would skip setting its own kernels' shared-memory attribute.
namespace {

constexpr int kMaxLaunchDevices = 64;

template <int BN, int STAGES, int ACC, int PAIR, typename OutT, int kFeat>
cudaError_t launch_gemm_t(const GemmLaunch& l) {
  using S = SmemLayout<BN, STAGES, PAIR, OutT>;
  constexpr size_t kSmem = sizeof(S) + 1024;
  static_assert(kSmem <= 232448, "shared memory budget");
  auto kern = grouped_gemm_kernel<BN, STAGES, ACC, PAIR, OutT, kFeat>;
  static bool attr_done[kMaxLaunchDevices] = {};
  if (l.device < 0 || l.device >= kMaxLaunchDevices) return cudaErrorInvalidDevice;
  if (!attr_done[l.device]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e == cudaSuccess && PAIR > 1) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e != cudaSuccess) return e;
    attr_done[l.device] = true;
  }
  const long long units = std::max(1LL, std::min<long long>(std::min(l.num_sms, kMaxGridCtas) / PAIR, l.max_units));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(units * PAIR), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = l.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: the GEMM may start while the scale-pack
  // kernel that precedes it still runs (that kernel lets it go at once); its
  // roles that read what the pack writes wait for it with griddepcontrol.wait.
  // After any other kernel, which never lets it go early, this changes nothing.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, l.maps->a, l.maps->a_self, l.maps->b, l.maps->out, *l.params);
}

template <int BN, int STAGES, int ACC, int PAIR, int kFeat>
cudaError_t launch_gemm_out(const GemmLaunch& l) {
  switch (l.out_dtype) {
    case MXGG_DTYPE_F16: return launch_gemm_t<BN, STAGES, ACC, PAIR, __half, kFeat>(l);
    case MXGG_DTYPE_F32: return launch_gemm_t<BN, STAGES, ACC, PAIR, float, kFeat>(l);
    default: return launch_gemm_t<BN, STAGES, ACC, PAIR, __nv_bfloat16, kFeat>(l);
  }
}

// Tile shapes: a CTA pair per 256 x BN tile (6 stages of 256 x 128, 8 of
// 256 x 128 for BN 128) or one CTA per 128 x BN tile (4 / 6 stages).
template <int kFeat>
cudaError_t launch_gemm_build(const GemmLaunch& l) {
  if (l.pair == 2) {
    if (l.bn == 256) return launch_gemm_out<256, 6, 2, 2, kFeat>(l);
    return launch_gemm_out<128, 8, 2, 2, kFeat>(l);
  }
  if (l.bn == 256) return launch_gemm_out<256, 4, 2, 1, kFeat>(l);
  return launch_gemm_out<128, 6, 2, 1, kFeat>(l);
}

}  // namespace
}  // namespace mxgg
