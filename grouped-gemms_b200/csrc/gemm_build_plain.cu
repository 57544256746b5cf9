// Grouped-GEMM build: 0 (see kFeat* in grouped_gemm.cuh).
#include "gemm_build.cuh"

namespace mxgg {

cudaError_t launch_gemm_plain(const GemmLaunch& l) { return launch_gemm_build<0>(l); }

}  // namespace mxgg
