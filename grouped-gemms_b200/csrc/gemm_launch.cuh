// Launch entry points of the grouped-GEMM kernel builds.  Each build (a mask
// of optional paths, see kFeat* in grouped_gemm.cuh) is instantiated in its
// own translation unit (gemm_build_*.cu), so the builds compile in parallel;
// capi.cu chooses one per call.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "grouped_gemm.cuh"

namespace mxgg {

// The grid never holds more CTAs than this (B200: 148 SMs); it bounds the
// split-tail scratch, which is therefore independent of the problem.
constexpr int kMaxGridCtas = 160;

struct Maps {
  CUtensorMap a, a_self, b;
  OutMaps out;
};

// One GEMM launch: tile columns bn (128 / 256) and CTAs per tile pair (1 / 2)
// pick the instantiation, out_dtype (MXGG_DTYPE_*) its output type.  Returns
// the CUDA error of the launch (cudaSuccess when queued).
struct GemmLaunch {
  int device;
  int num_sms;
  const Maps* maps;
  const GemmParams* params;
  long long max_units;
  int out_dtype;
  int bn;
  int pair;
  cudaStream_t stream;
};

cudaError_t launch_gemm_plain(const GemmLaunch& l);   // no optional path
cudaError_t launch_gemm_split(const GemmLaunch& l);   // kFeatSplit
cudaError_t launch_gemm_ep(const GemmLaunch& l);      // kFeatEp
cudaError_t launch_gemm_full(const GemmLaunch& l);    // every optional path

}  // namespace mxgg
