// Expert parallelism over NVLink peer memory: the end of a layer call whose output rows went
// straight into the owning ranks' receive buffers (OutMap, written by the GEMM2 and combine
// epilogues of this call).
//
// Every rank holds all T tokens and E/N experts; rank r owns tokens [r*shard, (r+1)*shard).
// Receive buffer of rank r: bf16 [2 phases][N slots][shard][7168]; slot j holds rank j's
// contribution to rank r's tokens.  Flags of rank r: uint32 [2 phases][kMaxRanks]; flag j of
// phase p holds the epoch of the last call in which rank j completed its rows for r.
//
//   ep_signal_kernel  after the layer's kernels (stream order: their stores have been
//                     performed), a system-scope fence, then lane r stores this call's epoch
//                     into rank r's flag [phase][this rank] with release semantics.
//   ep_reduce_kernel  waits (bounded by EpArgs::wait_ns) until all N flags of this rank's phase read this epoch,
//                     then sums the N slots row by row in rank order (fp32, one bf16 rounding)
//                     into this rank's shard.
//
// Two phases (epoch parity) keep a rank from overwriting rows a peer is still reading: before
// rank j writes call e's rows, its call e-1 waited for every rank's call e-1 flag, so every
// rank has finished reading phase(e-2) = phase(e).  Within a call the result depends only on
// the slots, summed in rank order, so it is deterministic.
#include <cuda_bf16.h>

#include "launch_args.cuh"
#include "moe_internal.cuh"
#include "ptx.cuh"

namespace moe {

constexpr int kEpThreads = 256;

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void ep_signal_kernel(EpArgs a) {
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < a.world) st_release_sys(a.signal[r] + a.phase * kMaxRanks + a.rank, a.epoch);
}

__global__ void __launch_bounds__(kEpThreads) ep_reduce_kernel(EpArgs a) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned int* flags = a.signal[a.rank] + a.phase * kMaxRanks;
    const uint64_t t0 = globaltimer_ns();
    int ok = 1;
    for (int j = 0; j < a.world && ok; ++j) {
      for (uint32_t i = 0; ld_acquire_sys(flags + j) != a.epoch; ++i) {
        if ((i & 63u) == 63u && globaltimer_ns() - t0 > a.wait_ns) {
          atomicCAS(a.status, 0, kStWaitPeers);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();   // the acquire above orders every thread's reads after the peers' rows
  if (!s_ok) return;
  const size_t slot = static_cast<size_t>(a.shard) * kH;   // bf16 elements of one slot
  const size_t n8 = slot / 8;
  for (size_t i = static_cast<size_t>(blockIdx.x) * kEpThreads + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * kEpThreads) {
    uint4 v[kMaxRanks];
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j)
      if (j < a.world) v[j] = __ldcg(reinterpret_cast<const uint4*>(a.recv + j * slot) + i);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      if (j >= a.world) break;
      const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[2 * k] = __fadd_rn(acc[2 * k], __uint_as_float(w[k] << 16));
        acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], __uint_as_float(w[k] & 0xFFFF0000u));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
      o[k] = *reinterpret_cast<uint32_t*>(&b);
    }
    reinterpret_cast<uint4*>(a.out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t ep_finish_launch(const EpArgs& a, int sms, cudaStream_t st, int* launches) {
  ep_signal_kernel<<<1, 32, 0, st>>>(a);
  ++*launches;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t n8 = static_cast<size_t>(a.shard) * kH / 8;
  const size_t want = (n8 + kEpThreads - 1) / kEpThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(4 * sms) ? want : static_cast<size_t>(4 * sms));
  ep_reduce_kernel<<<grid > 0 ? grid : 1, kEpThreads, 0, st>>>(a);
  ++*launches;
  return cudaGetLastError();
}

}  // namespace moe
