// Grouped-GEMM build: kFeatSplit | kFeatEp | kFeatQuant | kFeatAcc (see kFeat* in grouped_gemm.cuh).
#include "gemm_build.cuh"

namespace mxgg {

cudaError_t launch_gemm_full(const GemmLaunch& l) {
  return launch_gemm_build<kFeatSplit | kFeatEp | kFeatQuant | kFeatAcc>(l);
}

}  // namespace mxgg
