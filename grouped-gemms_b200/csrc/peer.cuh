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
// goes to rows [32 * rb, 32 * rb + 32) of the row-major output.  One warp
// per block, four passes: in pass i lane l moves the block's 16-byte piece
// q = 32 i + l (row q / 4), so every load is 512 contiguous bytes and every
// store covers eight rows with whole 64-byte runs (full 32-byte sectors).
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
    const uint4* src = reinterpret_cast<const uint4*>(inbox + (rb * chunks + cc) * 2048);
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __ldcs(src + 32 * i + lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = 32 * i + lane;
      const int r = q >> 2;
      const int j = (q & 3) ^ ((r >> 1) & 3);
      *reinterpret_cast<uint4*>(out + (rb * 32 + r) * row_bytes + (long long)cc * 64 + j * 16) = v[i];
    }
  }
}

// Sums the n replicas of a flat array that n GPUs hold, one copy each, in
// buffers this process has mapped (b.p[r]: replica r's buffer).  The replica
// running this kernel owns the 16-byte chunks [lo, hi): it loads each chunk
// from every replica (its own over HBM, the peers' over NVLink), adds them in
// fp32 in replica order 0, 1, ..., n - 1, rounds once to T and stores the sum
// into every replica.  The replicas own disjoint chunk ranges, so each
// element is summed once, in the same order, and every replica ends with the
// same bits.  Inputs are published before the launch and the sums after it
// by mxgg_peer_barrier over the replicas.
struct ReplicaBufs {
  uint8_t* p[kMaxDst];
};

template <typename T>
__device__ __forceinline__ float elem_to_float(T v);
template <>
__device__ __forceinline__ float elem_to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float elem_to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float elem_to_float<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T float_to_elem(float v);
template <>
__device__ __forceinline__ float float_to_elem<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 float_to_elem<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half float_to_elem<__half>(float v) { return __float2half_rn(v); }

template <typename T, int NR>
__global__ void __launch_bounds__(256) replica_sum_kernel(const ReplicaBufs b, long long lo, long long hi) {
  constexpr int kL = 16 / (int)sizeof(T);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long c = lo + (long long)blockIdx.x * blockDim.x + threadIdx.x; c < hi; c += stride) {
    uint4 v[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) v[r] = __ldcs(reinterpret_cast<const uint4*>(b.p[r]) + c);
    float acc[kL];
    {
      const T* e = reinterpret_cast<const T*>(&v[0]);
#pragma unroll
      for (int i = 0; i < kL; ++i) acc[i] = elem_to_float<T>(e[i]);
    }
#pragma unroll
    for (int r = 1; r < NR; ++r) {
      const T* e = reinterpret_cast<const T*>(&v[r]);
#pragma unroll
      for (int i = 0; i < kL; ++i) acc[i] += elem_to_float<T>(e[i]);
    }
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < kL; ++i) oe[i] = float_to_elem<T>(acc[i]);
#pragma unroll
    for (int r = 0; r < NR; ++r) __stcs(reinterpret_cast<uint4*>(b.p[r]) + c, o);
  }
}

template <typename T>
void launch_replica_sum(const ReplicaBufs& b, int n, long long lo, long long hi, unsigned blocks, cudaStream_t s) {
  switch (n) {
    case 2: replica_sum_kernel<T, 2><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    case 3: replica_sum_kernel<T, 3><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    case 4: replica_sum_kernel<T, 4><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    case 5: replica_sum_kernel<T, 5><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    case 6: replica_sum_kernel<T, 6><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    case 7: replica_sum_kernel<T, 7><<<blocks, 256, 0, s>>>(b, lo, hi); break;
    default: replica_sum_kernel<T, 8><<<blocks, 256, 0, s>>>(b, lo, hi); break;
  }
}

}  // namespace mxgg
