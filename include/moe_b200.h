/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) DeepSeek-V3 FP8 block-scale MoE layer.
 *
 * The layer is the contest definition
 * moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048 of the reference
 * (spec/definition.json:1-146).  Its Python entry point `run(...)` /
 * `kernel(...)` (spec/reference_official.py:5-16,
 * solution/python/kernel.py:1448-1459) is mirrored by moe_swarm_b200.run, which
 * calls moe_b200_forward below.  The reference's own native boundary was a
 * pybind11 module exporting gemm1 / gemm1_streaming / gemm2 over raw uintptr_t
 * pointers and a stream (solution/python/kernel.py:2497-2499, :2543-2551); this
 * header replaces it with one C entry point for the whole layer plus a
 * routing-only entry point for tests.
 *
 * Conventions: plain pointers to device memory, sizes in elements, the CUDA
 * stream passed as an opaque pointer (NULL = legacy default stream), integer
 * status codes (0 = success), no exceptions, no torch types.  All work is
 * enqueued on the stream without a host synchronisation, so calls can be
 * captured in a CUDA graph.  Device-side failures (a bounded wait that timed
 * out) are reported through moe_b200_device_status.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_B200_API __attribute__((visibility("default")))
#else
#define MOE_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Fixed DeepSeek-V3 geometry (spec/definition.json:8-54). */
#define MOE_B200_HIDDEN 7168
#define MOE_B200_INTER 2048
#define MOE_B200_EXPERTS 256
#define MOE_B200_TOPK 8

/* Status codes. */
#define MOE_B200_OK 0
#define MOE_B200_ERR_ARG 1         /* a null pointer, a bad size or an unsupported E_local */
#define MOE_B200_ERR_WORKSPACE 2   /* workspace too small (see moe_b200_workspace_size) */
#define MOE_B200_ERR_CUDA 3        /* a CUDA runtime/driver call failed (see moe_b200_last_error) */
#define MOE_B200_ERR_DEVICE 4      /* an sm_100 device is required */
#define MOE_B200_ERR_TIMEOUT 5     /* a device-side bounded wait gave up (device status) */

/*
 * Arguments of one layer call.  Tensor layouts are exactly those of
 * spec/definition.json:57-145 (all row-major, contiguous):
 *   routing_logits       f32  [T, 256]
 *   routing_bias         bf16 [256]                 (raw 16-bit words)
 *   hidden_states        e4m3 [T, 7168]             (raw bytes)
 *   hidden_states_scale  f32  [56, T]               (transposed per-token 1x128 scales)
 *   gemm1_weights        e4m3 [E_local, 4096, 7168]
 *   gemm1_weights_scale  f32  [E_local, 32, 56]
 *   gemm2_weights        e4m3 [E_local, 7168, 2048]
 *   gemm2_weights_scale  f32  [E_local, 56, 16]
 *   output               bf16 [T, 7168]             (written in full)
 * E_local may be any value in [1, 256]; the reference fixes it to 32
 * (spec/reference_official.py:44) and treats other values as expert
 * parallelism by local_expert_offset (reference/kernel_pytorch_v1.py:126-130).
 * The weight base pointers must be 16-byte aligned (TMA).
 */
typedef struct moe_b200_args {
  const float* routing_logits;
  const uint16_t* routing_bias;
  const uint8_t* hidden_states;
  const float* hidden_states_scale;
  const uint8_t* gemm1_weights;
  const float* gemm1_weights_scale;
  const uint8_t* gemm2_weights;
  const float* gemm2_weights_scale;
  uint16_t* output;
  int32_t num_tokens;            /* T >= 0 */
  int32_t num_local_experts;     /* E_local */
  int32_t local_expert_offset;   /* global id of local expert 0 */
  float routed_scaling_factor;
} moe_b200_args;

/*
 * Byte offsets of the per-call buffers inside a workspace, for tests and
 * tools that read the routing results back.  Arrays sized by T are laid out
 * for the T passed to moe_b200_workspace_layout.
 */
typedef struct moe_b200_layout {
  size_t plan;        /* int32[8]: T, E_local, rows, 128-row token tiles, 32-row token tiles */
  size_t topk_idx;    /* int32 [T, 8]: selected global experts, ascending per token */
  size_t topk_w;      /* f32   [T, 8]: their combine weights (bias-free, normalised, x rsf) */
  size_t tok_nloc;    /* int32 [T]: number of local experts each token selected */
  size_t tok_rows;    /* int32 [T, 8]: permuted row of each local pick, ascending expert */
  size_t e_count;     /* int32 [E_local]: rows per local expert */
  size_t e_start;     /* int32 [E_local + 1]: first permuted row of each local expert */
  size_t row_token;   /* int32 [R]: token of each permuted row (expert-major, token-minor) */
  size_t row_weight;  /* f32   [R]: combine weight of each permuted row */
  size_t c_hi;        /* e4m3  [R, 2048]: SwiGLU output, high part */
  size_t c_lo;        /* e4m3  [R, 2048]: SwiGLU output, residual x16 */
  size_t c_scale;     /* f32   [16, r_pad]: per-(row, 128-block) scale of c_hi */
  size_t status;      /* int32: device status word (0 = ok) */
  size_t trace;       /* uint64 [4 kernels][256 CTAs][16]: per-CTA counters of a traced build */
  size_t r_max;       /* rows reserved: T * min(8, E_local) */
  size_t r_pad;       /* leading dimension of the [blocks, rows] scale arrays */
  size_t total;       /* bytes */
} moe_b200_layout;

/* Workspace bytes one call with this T and E_local needs (0 on bad arguments).  Every entry point
 * that takes a workspace requires it 256-byte aligned (cudaMalloc's alignment); others return
 * MOE_B200_ERR_ARG. */
MOE_B200_API size_t moe_b200_workspace_size(int32_t num_tokens, int32_t num_local_experts);

/* Fills *out with the layout for (T, E_local).  Returns a status code. */
MOE_B200_API int moe_b200_workspace_layout(int32_t num_tokens, int32_t num_local_experts,
                              moe_b200_layout* out);

/*
 * Zeroes the self-resetting counters and the status word of a freshly
 * allocated workspace.  Call once after allocating (or after a call that
 * returned an error); later calls leave the counters zeroed themselves.
 */
MOE_B200_API int moe_b200_workspace_init(void* workspace, size_t workspace_bytes, int32_t num_tokens,
                            int32_t num_local_experts, void* stream);

/*
 * One MoE layer call: routing, permutation, GEMM1 + SwiGLU, GEMM2 + weighted
 * combine, bf16 output.  Replaces the whole of kernel(...)
 * (solution/python/kernel.py:1448-1538) and run(...)
 * (spec/reference_official.py:5-168).
 */
MOE_B200_API int moe_b200_forward(const moe_b200_args* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * The layer with the routing given by the caller instead of computed from logits: token t's
 * experts are topk_idx[t, 0..7] (global ids, distinct per token) with combine weights
 * topk_w[t, 0..7] (routed_scaling_factor already applied); routing_logits, routing_bias and
 * routed_scaling_factor of `args` are not read.  Otherwise as moe_b200_forward.  For
 * token-dispatch expert parallelism, where a rank receives tokens routed elsewhere.  It
 * replaces the routing half of the reference's kernel(...) (solution/python/kernel.py:137-213);
 * the rest of the call is the same.
 */
MOE_B200_API int moe_b200_forward_routed(const moe_b200_args* args, const int32_t* topk_idx,
                                         const float* topk_w, void* workspace, size_t workspace_bytes,
                                         void* stream);

/*
 * Expert parallelism over NVLink peer memory (no counterpart in the reference, whose layer is
 * one GPU's; it replaces the layer call followed by a separate reduce-scatter).  N ranks each
 * hold all T tokens (T a multiple of N) and their own E_local experts (`args`, as for
 * moe_b200_forward; args->output is not written).  Rank r owns tokens
 * [r*shard_tokens, (r+1)*shard_tokens).  The GEMM2 and combine epilogues store every output row
 * of this rank straight into the owning rank's receive buffer, in this rank's slot.  Each rank
 * then waits (bounded; a timeout sets the device status) for the N slots of its tokens and
 * sums them in rank order, in fp32 with one bf16 rounding, into out_shard.
 *
 * recv[r] and signal[r] are rank r's buffers, mapped in this process (e.g. torch symmetric
 * memory): recv bf16 [2][N][shard_tokens][7168], signal uint32 [2][8], zeroed once before the
 * first call.  `epoch` counts the calls 1, 2, 3, ..., the same on every rank; its parity
 * selects the half of both buffers this call uses.  Every rank makes every call.
 */
#define MOE_B200_MAX_RANKS 8
typedef struct moe_b200_ep {
  int32_t world;                          /* N, 1..8 */
  int32_t rank;                           /* this rank, 0..N-1 */
  int32_t shard_tokens;                   /* T / N */
  uint32_t epoch;                         /* call number, from 1 */
  void* recv[MOE_B200_MAX_RANKS];         /* per rank: its receive buffer */
  uint32_t* signal[MOE_B200_MAX_RANKS];   /* per rank: its flag words */
  void* out_shard;                        /* this rank's result, bf16 [shard_tokens][7168] */
  uint32_t wait_limit_us;                 /* bound of the wait for the peers' rows in
                                             microseconds; 0 selects the default, 2 s.  When it
                                             runs out the call's kernels return and the device
                                             status reads 0x107 (moe_b200_device_status). */
} moe_b200_ep;
MOE_B200_API int moe_b200_forward_ep(const moe_b200_args* args, const moe_b200_ep* ep, void* workspace,
                                     size_t workspace_bytes, void* stream);

/*
 * Routing and permutation only (the reference's _route_kernel + _pf_permute_kernel,
 * solution/python/kernel.py:137-213, :1211-1243): fills the routing arrays of the
 * layout and zeroes output rows of tokens with no local expert.
 */
MOE_B200_API int moe_b200_route(const moe_b200_args* args, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * Routing and permutation metadata with no workspace at all (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they call in: inference
 * engines whose plugin/enqueue path forbids allocations because all device memory is planned
 * up front, and latency-critical paths that cannot afford cudaMalloc's implicit device-wide
 * synchronisation.  The scratch lives in a fixed 64 KB device array inside the library, so:
 *   - num_tokens must be <= 256 (larger batches get MOE_B200_ERR_ARG; use moe_b200_route with
 *     a workspace); num_local_experts <= 256;
 *   - every call on a device shares that array: calls that overlap on the GPU (two streams or
 *     two host threads on one device) race and must be serialised by the caller;
 *   - the first call on a device looks up the array's device address (once per device, with
 *     that device current) and keeps it for the life of the process; a cudaDeviceReset of that
 *     device in the calling process invalidates the kept address, so make no call on a device
 *     after resetting it;
 * Only routing_logits, routing_bias, num_tokens, num_local_experts, local_expert_offset and
 * routed_scaling_factor of `args` are read.  Outputs (device memory, caller-allocated):
 *   topk_idx      int32 [T, 8]  selected global experts, ascending per token
 *   topk_w        f32   [T, 8]  their combine weights
 *   expert_count  int32 [E_local]  rows per local expert
 *   row_token     int32 [T * min(8, E_local)]  token of each permuted row (expert-major)
 *   row_weight    f32   [T * min(8, E_local)]  combine weight of each permuted row
 * Results equal moe_b200_route's.  Nothing is allocated; no host synchronisation.
 */
MOE_B200_API int moe_b200_route_noalloc(const moe_b200_args* args, int32_t* topk_idx, float* topk_w,
                                        int32_t* expert_count, int32_t* row_token, float* row_weight,
                                        void* stream);

/*
 * Synchronises the stream and returns the device status word (0 = ok,
 * otherwise the code of the first bounded wait that timed out); with
 * `clear` != 0 the word is reset.
 */
MOE_B200_API int moe_b200_device_status(void* workspace, size_t workspace_bytes, int32_t num_tokens,
                           int32_t num_local_experts, void* stream, int32_t clear);

/*
 * Per-stage device timing for benchmarks.  A timer records CUDA events on the
 * call's stream between the stages of moe_b200_forward_timed (routing +
 * permutation, GEMM1, GEMM2) and accumulates their durations; reading it
 * synchronises on the last recorded event.  Up to 4096 calls are held between
 * reads.  Timing adds two event records per stage and nothing else.
 */
typedef struct moe_b200_timer moe_b200_timer;
MOE_B200_API moe_b200_timer* moe_b200_timer_create(void);
MOE_B200_API void moe_b200_timer_destroy(moe_b200_timer* timer);
MOE_B200_API int moe_b200_forward_timed(const moe_b200_args* args, void* workspace,
                                        size_t workspace_bytes, void* stream, moe_b200_timer* timer);
/* stage_ms[3] = summed milliseconds of {routing+permutation, GEMM1, GEMM2}; *calls = calls
 * summed; with `reset` != 0 the timer is emptied.  Returns a status code. */
MOE_B200_API int moe_b200_timer_read(moe_b200_timer* timer, float* stage_ms, int32_t* calls,
                                     int32_t reset);

/* Text of the last host-side error of this thread ("" if none). */
MOE_B200_API const char* moe_b200_last_error(void);

/* Number of kernels the last moe_b200_forward call on this thread enqueued. */
MOE_B200_API int moe_b200_last_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
