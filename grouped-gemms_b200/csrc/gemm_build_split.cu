// Grouped-GEMM build: kFeatSplit (see kFeat* in grouped_gemm.cuh).
#include "gemm_build.cuh"

namespace mxgg {

cudaError_t launch_gemm_split(const GemmLaunch& l) { return launch_gemm_build<kFeatSplit>(l); }

}  // namespace mxgg
