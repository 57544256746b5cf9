// Grouped-GEMM build: kFeatEp (see kFeat* in grouped_gemm.cuh).
#include "gemm_build.cuh"

namespace mxgg {

cudaError_t launch_gemm_ep(const GemmLaunch& l) { return launch_gemm_build<kFeatEp>(l); }

}  // namespace mxgg
