// Expert-ordered combine of tokens routed to more than one local expert:
//   out[t, :] = bf16( sum over t's local experts, ascending, of w_e * O_e[t, :] )
// where the GEMM2 kernels left each w_e * O_e row in fp32 in the partial-row buffer.  This is
// the accumulation order of the reference's per-expert index_add_
// (spec/reference_official.py:134-166), so the result is deterministic.  Tokens with one local
// expert were written by GEMM2 directly; tokens with none get their zero row here.
#include <cuda_bf16.h>

#include "launch_args.cuh"
#include "moe_internal.cuh"
#include "ptx.cuh"

namespace moe {

static_assert(kCombineChunks * kCombineThreads * 4 == kH, "a row is a whole number of chunks");

// Work item i = (token i / 7, chunk i % 7): each thread owns one float4 of the chunk, so a
// token's partial rows are read in one round of independent loads, and at decode sizes the
// row's chunks spread over seven SMs.

__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const int* tok_nloc, const int* tok_rows,
                                                                  const float* part2, OutMap out, int T,
                                                                  unsigned long long* trace) {
  MOE_TRACE_CTA(trace, 0);
  pdl_wait();   // the partial rows come from GEMM2
  MOE_TRACE_CTA(trace, 2);
  for (int i = blockIdx.x; i < T * kCombineChunks; i += gridDim.x) {
    const int t = i / kCombineChunks;
    const int v = (i - t * kCombineChunks) * kCombineThreads + threadIdx.x;   // float4 index in the row
    const int kt = __ldg(tok_nloc + t);
    if (kt == 1) continue;
    if (kt == 0) {   // no local expert: this thread's 4 bf16 of the zero row
      reinterpret_cast<uint2*>(out_row(out, t))[v] = make_uint2(0, 0);
      continue;
    }
    int rows[kTopK];
#pragma unroll
    for (int a = 0; a < kTopK; ++a) rows[a] = a < kt ? __ldg(tok_rows + static_cast<size_t>(t) * kTopK + a) : 0;
    {
      float4 x[kTopK];
#pragma unroll
      for (int a = 0; a < kTopK; ++a)
        if (a < kt) x[a] = __ldcg(reinterpret_cast<const float4*>(part2 + static_cast<size_t>(rows[a]) * kH) + v);
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int a = 0; a < kTopK; ++a)
        if (a < kt) {
          s.x = __fadd_rn(s.x, x[a].x);
          s.y = __fadd_rn(s.y, x[a].y);
          s.z = __fadd_rn(s.z, x[a].z);
          s.w = __fadd_rn(s.w, x[a].w);
        }
      __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
      uint2 pk = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
      *reinterpret_cast<uint2*>(out_row(out, t) + 4 * v) = pk;
    }
  }
  (void)trace;
  MOE_TRACE_CTA(trace, 1);
}

// Launched as a programmatic dependent of GEMM2.
cudaError_t combine_launch(int T, int grid, cudaStream_t st, const int* tok_nloc, const int* tok_rows,
                           const float* part2, const OutMap& out, unsigned long long* trace) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_kernel, tok_nloc, tok_rows, part2, out, T, trace);
}

}  // namespace moe
