// Cross-GPU signalling for the expert-parallel path.
//
// peer_barrier_kernel: every rank writes `epoch` into slot `rank` of every
// rank's flag array (NVLink stores, release at system scope) and then waits
// until all `world` slots of its own array have reached `epoch` (acquire).
// It runs as one small kernel per GPU, ordered on the stream after the work
// it publishes (peer copies, the GEMM's peer stores) and before the work that
// consumes what the peers published.  The wait is bounded (wait_ns of
// %globaltimer, 1 s by default); a timeout sets kErrPeerWait in the status
// word and returns.
#pragma once

#include <cstdint>

#include "grouped_gemm.cuh"
#include "ptx.cuh"

namespace mxgg {

constexpr uint32_t kErrPeerWait = 64u;

struct PeerFlags {
  int* flags[kMaxDst];   // flags[r]: rank r's flag array (world ints), mapped into this process
};

__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerFlags f, int world, int rank, int epoch,
                                                          uint32_t* status, unsigned long long wait_ns) {
  const int t = threadIdx.x;
  // everything this stream did before (earlier kernels, copies) precedes the signal
  __threadfence_system();
  __syncwarp();
  if (t < world) {
    int* dst = f.flags[t] + rank;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
  }
  if (t < world) {
    const int* src = f.flags[rank] + t;
    const uint64_t t0 = ptx::globaltimer();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
      if (v - epoch >= 0) break;   // epochs only grow
      if (ptx::globaltimer() - t0 > wait_ns) {
        atomicOr(status, kErrPeerWait);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncwarp();
  __threadfence_system();
}

// Unpacks this rank's inbox: for each listed 32-row block and each 64-byte
// column chunk, the 2 KB block (rows in the 64-byte swizzle of the GEMM's
// staging buffer: row r's chunk j at r * 64 + (j ^ ((r >> 1) & 3)) * 16)
// goes to rows [32 * rb, 32 * rb + 32) of the row-major output.  One warp per
// block; consecutive warps take consecutive chunks of a row block, so each
// output line is completed in L2 before it is written back.
__global__ void __launch_bounds__(256) inbox_unpack_kernel(const uint8_t* __restrict__ inbox,
                                                           uint8_t* __restrict__ out,
                                                           const int32_t* __restrict__ row_blocks, int n_rb,
                                                           int chunks, long long row_bytes) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long total = (long long)n_rb * chunks;
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nwarps) {
    const int rbi = (int)(w / chunks);
    const int cc = (int)(w - (long long)rbi * chunks);
    const long long rb = __ldg(row_blocks + rbi);
    const uint4* src = reinterpret_cast<const uint4*>(inbox + (rb * chunks + cc) * 2048) + lane * 4;
    uint4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __ldcs(src + j);
    uint4* dst = reinterpret_cast<uint4*>(out + (rb * 32 + lane) * row_bytes + (long long)cc * 64);
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j ^ sw] = v[j];
  }
}

}  // namespace mxgg
