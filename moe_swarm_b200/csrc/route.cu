// DeepSeek-V3 no-aux routing fused with the token->expert histogram, the prefix sums
// (expert segments and GEMM tile tables) and the permutation into expert-major order: the row
// metadata always, and for the token-major GEMMs (T > 512) the activation rows and their scales
// copied into the workspace (the streaming GEMM1 gathers its rows from hidden_states itself).
//
// Semantics follow spec/reference_official.py:95-126 (selection on sigmoid(logits)+bias,
// 8 groups scored by their top-2 sum, 4 groups kept, top-8 experts, bias-free weights
// normalised then scaled) and the row order of reference/kernel_pytorch_v1.py:100-123
// (stable sort by local expert: expert-major, token-minor).  The reference's Triton kernel
// appends picks to per-expert buckets with atomics (solution/python/kernel.py:137-213),
// which makes the row order run-dependent; here every row index is a prefix count, so the
// permutation is deterministic and identical to the oracle's.
//
// route_kernel: one warp per token (lane l owns experts 8l..8l+7, the four lanes 4g..4g+3
// own group g), 8 tokens per CTA.  Local picks are counted per 128-token chunk with global
// atomics (order-independent sums).  The last CTA to finish (a self-resetting arrival
// counter) turns the chunk counts into expert segment starts, per-chunk bases and the GEMM
// tile tables (plan) and zeroes the counts for the next call.  scatter_kernel (a programmatic
// dependent of route_kernel): 8 tokens per CTA; the rank of a token in an expert's segment is
// a popcount over the chunk's per-expert token bitmask plus the chunk base.  At decode sizes
// one CTA does all of it in one launch with the pick lists and counts in shared memory.  Each
// routing CTA first starts its tokens' hidden rows and scales toward L2, so the permutation's
// copies (or GEMM1's gathers) find them there.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "../../include/moe_b200.h"
#include "launch_args.cuh"
#include "moe_internal.cuh"
#include "ptx.cuh"

namespace moe {

__device__ __forceinline__ uint32_t orderable(float v) {
  uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ int warp_excl_prefix(int v, int lane) {
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  return x - v;
}

// exp(y) rounded once to fp32, computed in double: y = k*ln2 + r with k = rint(y / ln2) and a
// two-part ln2 (fdlibm's split, k*ln2_hi exact), exp(r) for |r| <= ln2/2 by its Taylor series
// to degree 13 (truncation below 5e-18, under double rounding), then scaled by 2^k through the
// exponent field.  For every fp32 argument the result equals the library's double exp rounded
// to fp32 (checked exhaustively on a B200: all 2,246,049,794 floats with |x| <= 120 give the
// same bits; beyond that both saturate to +inf or 0).  About 20 double operations, several
// times fewer than the library's general double exp, which dominated the routing time.
__device__ __forceinline__ float exp_to_f32(double y) {
  if (y != y) return static_cast<float>(y);
  if (y > 100.0) return __int_as_float(0x7f800000);   // above FLT_MAX: +inf
  if (y < -110.0) return 0.f;                         // below half the smallest denormal
  const double k = rint(y * 1.4426950408889634074);
  double r = fma(-k, 6.93147180369123816490e-01, y);
  r = fma(-k, 1.90821492927058770002e-10, r);
  double p = 1.0 / 6227020800.0;
  p = fma(p, r, 1.0 / 479001600.0);
  p = fma(p, r, 1.0 / 39916800.0);
  p = fma(p, r, 1.0 / 3628800.0);
  p = fma(p, r, 1.0 / 362880.0);
  p = fma(p, r, 1.0 / 40320.0);
  p = fma(p, r, 1.0 / 5040.0);
  p = fma(p, r, 1.0 / 720.0);
  p = fma(p, r, 1.0 / 120.0);
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  const double scale = __hiloint2double((static_cast<int>(k) + 1023) << 20, 0);
  return static_cast<float>(p * scale);
}

// Where routing leaves each token's local picks for the permutation: global memory when the
// permutation is a separate launch (scatter_kernel), shared memory when one CTA does both.
struct PickBuf {
  int* le;     // [T][8] local expert ids, ascending
  float* lw;   // [T][8] their combine weights
  int* nloc;   // [T] local pick counts (also written to RouteArgs::tok_nloc for the combine)
  int* hist;   // [nchunks][E] per-chunk counts of local picks
};

__device__ __forceinline__ PickBuf global_picks(const RouteArgs& a) {
  return PickBuf{a.tok_le, a.tok_lw, a.tok_nloc, a.chunk_hist};
}

// Starts tokens [t0, t0 + nt) on their way to L2: their logits rows and, in the layer call,
// their hidden rows and 56 scales -- so the scatter's copies (and the streaming GEMM1's row
// gathers) find them in L2 rather than HBM once the routing, which needs only the logits, is done.
__device__ void prefetch_tokens(const RouteArgs& a, int t0, int nt, int tid, int nthr) {
  if (nt <= 0) return;
  if (a.logits) {
    const char* lg = reinterpret_cast<const char*>(a.logits + static_cast<size_t>(t0) * kEG);
    for (int i = tid; i < nt * (kEG * 4 / 128); i += nthr) prefetch_l2(lg + static_cast<size_t>(i) * 128);
  }
  if (!a.hidden) return;   // (rows are copied by the scatter, or gathered by the streaming GEMM1)
  const uint8_t* h = a.hidden + static_cast<size_t>(t0) * kH;
  for (int i = tid; i < nt * (kH / 128); i += nthr) prefetch_l2(h + static_cast<size_t>(i) * 128);
  // scales [56][T]: the run of nt floats of each K-block, its first and last line
  for (int i = tid; i < 2 * kKB1; i += nthr) {
    const int kb = i >> 1;
    prefetch_l2(a.hs_scale + static_cast<size_t>(kb) * a.T + t0 + ((i & 1) ? nt - 1 : 0));
  }
}

// Routes token t with the calling warp: writes its top-8 (ascending expert id) with weights,
// its local picks (ascending local expert) and their count, and adds the local picks to the
// token's chunk histogram.
// Phase times of the first routed token (traced builds): slots 6.. of CTA 0's routing record.
#ifdef MOE_TRACE
#define MOE_RT_MARK(i)                                                                         \
  do {                                                                                         \
    if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) a.trace[6 + (i)] = globaltimer_ns(); \
  } while (0)
#else
#define MOE_RT_MARK(i) (void)0
#endif

__device__ void route_token(const RouteArgs& a, const PickBuf& pb, const float* s_bias, int t, int lane) {
  MOE_RT_MARK(0);
  const float* lg = a.logits + static_cast<size_t>(t) * kEG + lane * 8;
  const float4 v0 = *reinterpret_cast<const float4*>(lg);
  const float4 v1 = *reinterpret_cast<const float4*>(lg + 4);
  const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  float s[8], sb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // sigmoid as 1/(1+exp(-x)) in fp32 (reference_official.py:99) with exp(-x) rounded
    // once to fp32 from a double evaluation (the correctly rounded fp32 exponential).
    const float e = exp_to_f32(-static_cast<double>(x[i]));
    s[i] = __frcp_rn(1.0f + e);   // correctly rounded 1 / (1 + e): the IEEE quotient, bit for bit
    sb[i] = s[i] + s_bias[lane * 8 + i];
  }
  MOE_RT_MARK(1);
  // group score: sum of the group's top-2 selection scores (multiset top-2)
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = sb[i];
    if (v > m1) {
      m2 = m1;
      m1 = v;
    } else if (v > m2) {
      m2 = v;
    }
  }
#pragma unroll
  for (int d = 1; d <= 2; d <<= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, m1, d);
    const float o2 = __shfl_xor_sync(0xffffffffu, m2, d);
    const float n1 = fmaxf(m1, o1);
    const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = n1;
    m2 = n2;
  }
  const float gscore = m1 + m2;
  const int g = lane >> 2;
  int rank = 0;
#pragma unroll
  for (int h = 0; h < kNGroup; ++h) {
    const float o = __shfl_sync(0xffffffffu, gscore, h * 4);
    rank += (o > gscore || (o == gscore && h < g)) ? 1 : 0;
  }
  const bool keep = rank < kTopKGroup;
  MOE_RT_MARK(2);
  // top-8 among the kept groups: 8 rounds of a warp-wide argmax (ties -> lower expert id).  Each
  // lane first sorts its 8 candidates descending by (key, lower slot first) with a 19-comparator
  // network on distinct composite keys; a round is then one warp max (redux), a ballot for the
  // lowest lane holding it, and a shift of the winning lane's list -- no rescan on the chain.
  uint64_t cand[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    cand[i] = (static_cast<uint64_t>(keep ? orderable(sb[i]) : 0u) << 3) | static_cast<uint64_t>(7 - i);
  auto cx = [&](int x, int y) {   // descending
    const uint64_t a = cand[x], b = cand[y];
    cand[x] = a > b ? a : b;
    cand[y] = a > b ? b : a;
  };
  cx(0, 2); cx(1, 3); cx(4, 6); cx(5, 7);
  cx(0, 4); cx(1, 5); cx(2, 6); cx(3, 7);
  cx(0, 1); cx(2, 3); cx(4, 5); cx(6, 7);
  cx(2, 4); cx(3, 5);
  cx(1, 4); cx(3, 6);
  cx(1, 2); cx(3, 4); cx(5, 6);
  uint32_t taken = 0;
#pragma unroll
  for (int r = 0; r < kTopK; ++r) {
    const uint32_t bkey = static_cast<uint32_t>(cand[0] >> 3);
    const uint32_t m = __reduce_max_sync(0xffffffffu, bkey);
    const uint32_t holders = __ballot_sync(0xffffffffu, bkey == m);
    if (lane == __ffs(holders) - 1) {
      taken |= 1u << (7 - static_cast<int>(cand[0] & 7u));
#pragma unroll
      for (int i = 0; i < 7; ++i) cand[i] = cand[i + 1];
      cand[7] = 0;
    }
  }
  MOE_RT_MARK(3);
  // combine weights from s (no bias): s / (sum + 1e-20) * rsf (reference_official.py:122-126)
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if ((taken >> i) & 1u) part += s[i];
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) part += __shfl_xor_sync(0xffffffffu, part, d);
  const float denom = part + 1e-20f;

  const int lo_g = a.offset, hi_g = a.offset + a.E;
  uint32_t local_mask = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ge = lane * 8 + i;
    if (((taken >> i) & 1u) && ge >= lo_g && ge < hi_g) local_mask |= 1u << i;
  }
  int pos = warp_excl_prefix(__popc(taken), lane);
  int lpos = warp_excl_prefix(__popc(local_mask), lane);
  int* idx_out = a.topk_idx + static_cast<size_t>(t) * kTopK;
  float* w_out = a.topk_w + static_cast<size_t>(t) * kTopK;
  int* le_out = pb.le + static_cast<size_t>(t) * kTopK;
  float* lw_out = pb.lw + static_cast<size_t>(t) * kTopK;
  int* hist = pb.hist + static_cast<size_t>(t / kChunk) * a.E;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if ((taken >> i) & 1u) {
      const int ge = lane * 8 + i;
      const float w = (s[i] / denom) * a.rsf;
      idx_out[pos] = ge;
      w_out[pos] = w;
      ++pos;
      if ((local_mask >> i) & 1u) {
        const int le = ge - lo_g;
        le_out[lpos] = le;
        lw_out[lpos] = w;
        ++lpos;
        atomicAdd(hist + le, 1);
      }
    }
  }
  int nloc = __popc(local_mask);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) nloc += __shfl_xor_sync(0xffffffffu, nloc, d);
  if (lane == 0) {
    a.tok_nloc[t] = nloc;
    pb.nloc[t] = nloc;
  }
  MOE_RT_MARK(4);
}

// Pre-routed token t (moe_b200_forward_routed): the caller's 8 picks (global expert id and
// combine weight) take the place of the routing.  Lanes 0..7 hold the picks; the local ones are
// written in ascending expert order -- the row order of the permutation and the order of the
// combine's sum -- and counted in the token's chunk histogram.  A token's ids must be distinct.
__device__ void pick_token(const RouteArgs& a, const PickBuf& pb, int t, int lane) {
  int ge = -1;
  float w = 0.f;
  if (lane < kTopK) {
    ge = __ldg(a.pre_idx + static_cast<size_t>(t) * kTopK + lane);
    w = __ldg(a.pre_w + static_cast<size_t>(t) * kTopK + lane);
    a.topk_idx[static_cast<size_t>(t) * kTopK + lane] = ge;
    a.topk_w[static_cast<size_t>(t) * kTopK + lane] = w;
  }
  const bool local = lane < kTopK && ge >= a.offset && ge < a.offset + a.E;
  int rank = 0;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    const int gj = __shfl_sync(0xffffffffu, ge, j);
    const int lj = __shfl_sync(0xffffffffu, local ? 1 : 0, j);
    if (lj && (gj < ge || (gj == ge && j < lane))) ++rank;
  }
  if (local) {
    const int le = ge - a.offset;
    pb.le[static_cast<size_t>(t) * kTopK + rank] = le;
    pb.lw[static_cast<size_t>(t) * kTopK + rank] = w;
    atomicAdd(pb.hist + static_cast<size_t>(t / kChunk) * a.E + le, 1);
  }
  const int nloc = __popc(__ballot_sync(0xffffffffu, local));
  if (lane == 0) {
    a.tok_nloc[t] = nloc;
    pb.nloc[t] = nloc;
  }
}

// Per-expert token bitmask of chunk c, built by the whole CTA from the tokens' pick lists.
__device__ void build_chunk_masks(const RouteArgs& a, const PickBuf& pb, int c, uint32_t (*s_mask)[kChunk / 32]) {
  for (int i = threadIdx.x; i < a.E * (kChunk / 32); i += blockDim.x) (&s_mask[0][0])[i] = 0;
  __syncthreads();
  const int t0 = c * kChunk;
  const int nt = min(kChunk, a.T - t0);
  for (int i = threadIdx.x; i < nt * kTopK; i += blockDim.x) {
    const int tl = i / kTopK, p = i % kTopK;
    const int t = t0 + tl;
    if (p < pb.nloc[t]) {
      const int le = pb.le[static_cast<size_t>(t) * kTopK + p];
      atomicOr(&s_mask[le][tl >> 5], 1u << (tl & 31));
    }
  }
  __syncthreads();
}

// Scatters the local picks of token t (index tl in its chunk) with the calling warp: row
// indices, row metadata, the fp8 activation row and its 56 scales.  A token with no local
// expert gets a zero output row instead.
__device__ void scatter_token(const RouteArgs& a, const PickBuf& pb, int t, int tl, int lane,
                              const uint32_t (*s_mask)[kChunk / 32], const int* base) {
  const int k = pb.nloc[t];
  if (k == 0) {
    if (a.out == nullptr) return;
    uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(t) * kH);
    for (int j = lane; j < kH * 2 / 16; j += 32) dst[j] = make_uint4(0, 0, 0, 0);
    return;
  }
  int row = 0;
  if (lane < k) {
    const int le = pb.le[static_cast<size_t>(t) * kTopK + lane];
    const float w = pb.lw[static_cast<size_t>(t) * kTopK + lane];
    int rank = 0;
    for (int wd = 0; wd < (tl >> 5); ++wd) rank += __popc(s_mask[le][wd]);
    rank += __popc(s_mask[le][tl >> 5] & ((1u << (tl & 31)) - 1u));
    row = base[le] + rank;
    a.row_token[row] = t;
    a.row_weight[row] = w;
    if (a.row_nloc) a.row_nloc[row] = k;
    a.tok_rows[static_cast<size_t>(t) * kTopK + lane] = row;
  }
  int rows[kTopK];
#pragma unroll
  for (int i = 0; i < kTopK; ++i) rows[i] = __shfl_sync(0xffffffffu, row, i);
  if (a.a_perm == nullptr) return;   // routing metadata only
  // the 7 KB row moves in two halves of 7 independent 16-byte loads per lane (all loads
  // of a half issue before its stores)
  const uint4* src = reinterpret_cast<const uint4*>(a.hidden + static_cast<size_t>(t) * kH);
  constexpr int kVec = kH / 16 / 32 / 2;   // 7 uint4 per lane per half
  const float sc0 = a.hs_scale[static_cast<size_t>(lane) * a.T + t];
  const float sc1 = lane + 32 < kKB1 ? a.hs_scale[static_cast<size_t>(lane + 32) * a.T + t] : 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint4 v[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) v[j] = __ldg(src + lane + 32 * (j + kVec * half));
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
      if (i >= k) break;
      uint4* dst = reinterpret_cast<uint4*>(a.a_perm + static_cast<size_t>(rows[i]) * kH);
#pragma unroll
      for (int j = 0; j < kVec; ++j) dst[lane + 32 * (j + kVec * half)] = v[j];
    }
  }
#pragma unroll
  for (int i = 0; i < kTopK; ++i) {
    if (i >= k) break;
    a.sa_perm[static_cast<size_t>(lane) * a.r_pad + rows[i]] = sc0;
    if (lane + 32 < kKB1) a.sa_perm[static_cast<size_t>(lane + 32) * a.r_pad + rows[i]] = sc1;
  }
}

// Chunk counts -> expert segment starts, per-chunk bases, tile prefixes and the plan.
// Run by one whole CTA (blockDim >= 256).  `hist` / `cbase` are [nchunks][E]: in global memory
// (GLOBAL, filled by atomics of other CTAs; the counts are zeroed here for the next call) or
// in this CTA's shared memory.
template <bool GLOBAL>
__device__ void scan_plan(const RouteArgs& a, int* hist, int* cbase, int* s_tmp) {
  const int tid = threadIdx.x;
  const int E = a.E;
  auto rd = [&](size_t i) { return GLOBAL ? __ldcg(hist + i) : hist[i]; };
  int cnt = 0;
  int first[8] = {};   // the first eight chunks' counts, kept for the base pass below
  if (tid < E)
    for (int c0 = 0; c0 < a.nchunks; c0 += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = c0 + j < a.nchunks ? rd(static_cast<size_t>(c0 + j) * E + tid) : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cnt += v[j];
        if (c0 == 0) first[j] = v[j];
      }
    }
  // inclusive scans over experts (threads 0..255) of rows and of 128- and 32-row tiles: a
  // shuffle scan inside each warp, then each thread adds the totals of the warps before it
  const int lane = tid & 31, warp = tid >> 5;
  const int ucnt = tid < E ? cnt : 0;
  const int umt = (ucnt + kBlk - 1) / kBlk, utt = (ucnt + kTok - 1) / kTok;
  int x0 = ucnt, x1 = umt, x2 = utt;
  if (tid < 256) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y0 = __shfl_up_sync(0xffffffffu, x0, d);
      const int y1 = __shfl_up_sync(0xffffffffu, x1, d);
      const int y2 = __shfl_up_sync(0xffffffffu, x2, d);
      if (lane >= d) {
        x0 += y0;
        x1 += y1;
        x2 += y2;
      }
    }
    if (lane == 31) {
      s_tmp[warp] = x0;
      s_tmp[8 + warp] = x1;
      s_tmp[16 + warp] = x2;
    }
  }
  __syncthreads();
  int rows = 0, mtiles = 0, ttiles = 0;
  if (tid < 256) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int w0 = s_tmp[w], w1 = s_tmp[8 + w], w2 = s_tmp[16 + w];
      if (w < warp) {
        x0 += w0;
        x1 += w1;
        x2 += w2;
      }
      rows += w0;
      mtiles += w1;
      ttiles += w2;
    }
  }
  if (tid == 0) {
    Plan p{};
    p.T = a.T;
    p.E = E;
    p.rows = rows;
    p.m_tiles = mtiles;
    p.tt = ttiles;
    *a.plan = p;
  }
  if (tid < E) {
    const int start = x0 - cnt;
    a.e_count[tid] = cnt;
    a.e_start[tid] = start;
    a.e_mt_start[tid] = x1 - umt;
    a.e_tt[tid] = x2 - utt;
    int run = start;
    for (int c0 = 0; c0 < a.nchunks; c0 += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = c0 == 0 ? first[j] : c0 + j < a.nchunks ? rd(static_cast<size_t>(c0 + j) * E + tid) : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (c0 + j < a.nchunks) {
          cbase[static_cast<size_t>(c0 + j) * E + tid] = run;
          if (GLOBAL) hist[static_cast<size_t>(c0 + j) * E + tid] = 0;   // self-reset for the next call
        }
        run += v[j];
      }
    }
  }
  if (tid == 0) {
    a.e_start[E] = rows;
    a.e_mt_start[E] = mtiles;
    a.e_tt[E] = ttiles;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  __shared__ float s_bias[kEG];
  __shared__ int s_tmp[32];   // per-warp totals of the expert scans
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  MOE_TRACE_CTA(a.trace, 0);
  pdl_launch_dependents();   // scatter_kernel's CTAs may become resident meanwhile
  const int tb = blockIdx.x * kRouteWarps;
  prefetch_tokens(a, tb, min(kRouteWarps, a.T - tb), tid, blockDim.x);
  if (!a.pre_idx)   // pre-routed calls have no logits or bias
    for (int i = tid; i < kEG; i += blockDim.x) s_bias[i] = bf16_bits_to_float(a.bias[i]);
  __syncthreads();
  const PickBuf pb = global_picks(a);
  const int t = tb + warp;
  if (t < a.T) {
    if (a.pre_idx) pick_token(a, pb, t, lane);
    else route_token(a, pb, s_bias, t, lane);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(a.route_done, 1);
    s_last = (prev == static_cast<int>(gridDim.x) - 1);
  }
  __syncthreads();
  MOE_TRACE_CTA(a.trace, 1);
  if (!s_last) return;
  __threadfence();
  scan_plan<true>(a, a.chunk_hist, a.chunk_base, s_tmp);
  if (tid == 0) *a.route_done = 0;   // self-reset for the next call
  MOE_TRACE_CTA(a.trace, 1);
}

__global__ void __launch_bounds__(kRouteThreads) scatter_kernel(RouteArgs a) {
  __shared__ uint32_t s_mask[kEG][kChunk / 32];
  __shared__ int s_base[kEG];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long* tr = a.trace ? a.trace + kMaxSms * kTraceSlots : nullptr;
  MOE_TRACE_CTA(tr, 0);
  pdl_wait();                // the picks and the chunk bases come from route_kernel
  pdl_launch_dependents();   // GEMM1 may run its prologue meanwhile
  const PickBuf pb = global_picks(a);
  const int t0 = blockIdx.x * kRouteWarps;   // this CTA's tokens: t0 .. t0+7 (one chunk)
  const int c = t0 / kChunk;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) s_base[e] = a.chunk_base[static_cast<size_t>(c) * a.E + e];
  build_chunk_masks(a, pb, c, s_mask);
  const int t = t0 + warp;
  if (t < a.T) scatter_token(a, pb, t, t - c * kChunk, lane, s_mask, s_base);
  (void)tr;
  MOE_TRACE_CTA(tr, 1);
}

// T <= kRouteSmallT: one CTA routes every token (one warp each, a single round), scans and
// scatters in a single launch -- the decode regime, where a second launch would cost more than
// it saves.  Larger batches spread the tokens over T/8 CTAs (a warp's routing of one token is a
// serial chain of several thousand cycles, and one SM would take T/32 of them in turn) and
// permute with scatter_kernel on as many CTAs.
constexpr int kRouteSmallT = 32;
constexpr int kRouteSmallThreads = 1024;
// The one-CTA body for T <= MAXT (route_small_kernel: kRouteSmallT; the no-alloc entry point:
// kNoAllocMaxT).  Its pick lists, chunk counts and chunk bases live in shared memory, so the
// scan and the permutation read them without an L2 round trip; sized by MAXT so that the
// decode kernel leaves room on its SM for a GEMM CTA.
template <int MAXT>
__device__ __forceinline__ void route_small_body(const RouteArgs& a) {
  constexpr int kChunks = (MAXT + kChunk - 1) / kChunk;
  __shared__ float s_bias[kEG];
  __shared__ uint32_t s_mask[kEG][kChunk / 32];
  __shared__ int s_tmp[32];   // per-warp totals of the expert scans
  __shared__ int s_base[kEG];
  __shared__ int s_le[MAXT * kTopK];
  __shared__ float s_lw[MAXT * kTopK];
  __shared__ int s_nloc[MAXT];
  __shared__ int s_hist[kChunks * kEG];
  __shared__ int s_cbase[kChunks * kEG];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  prefetch_tokens(a, 0, a.T, tid, blockDim.x);
  if (!a.pre_idx)   // pre-routed calls have no logits or bias
    for (int i = tid; i < kEG; i += blockDim.x) s_bias[i] = bf16_bits_to_float(a.bias[i]);
  for (int i = tid; i < a.nchunks * a.E; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  MOE_TRACE_CTA(a.trace, 2);
  const PickBuf pb{s_le, s_lw, s_nloc, s_hist};
  for (int t = warp; t < a.T; t += kRouteSmallThreads / 32) {
    if (a.pre_idx) pick_token(a, pb, t, lane);
    else route_token(a, pb, s_bias, t, lane);
  }
  __syncthreads();
  MOE_TRACE_CTA(a.trace, 3);
  scan_plan<false>(a, s_hist, s_cbase, s_tmp);
  MOE_TRACE_CTA(a.trace, 4);
  for (int c = 0; c < a.nchunks; ++c) {
    for (int e = tid; e < a.E; e += blockDim.x) s_base[e] = s_cbase[c * a.E + e];
    build_chunk_masks(a, pb, c, s_mask);
    MOE_TRACE_CTA(a.trace, 5);
    const int t0 = c * kChunk, nt = min(kChunk, a.T - t0);
    for (int tl = warp; tl < nt; tl += kRouteSmallThreads / 32) scatter_token(a, pb, t0 + tl, tl, lane, s_mask, s_base);
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kRouteSmallThreads, 1) route_small_kernel(RouteArgs a) {
  MOE_TRACE_CTA(a.trace, 0);
  pdl_launch_dependents();   // the GEMM that follows may run its prologue meanwhile
  route_small_body<kRouteSmallT>(a);
  MOE_TRACE_CTA(a.trace, 1);
}

cudaError_t route_launch(const RouteArgs& a, cudaStream_t st, int* launches) {
  if (a.T <= kRouteSmallT) {
    route_small_kernel<<<1, kRouteSmallThreads, 0, st>>>(a);
    ++*launches;
    return cudaGetLastError();
  }
  const int grid = (a.T + kRouteWarps - 1) / kRouteWarps;
  route_kernel<<<grid, kRouteThreads, 0, st>>>(a);
  ++*launches;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // a programmatic dependent of route_kernel: its CTAs wait resident for the routing
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, scatter_kernel, a);
  ++*launches;
  return e;
}

// ---------------------------------------------------------------------------------------
// Routing without a caller-provided workspace (moe_b200_route_noalloc).
//
// Its scratch -- the per-token local pick counts and row lists, the segment tables and the plan
// -- lives in this file-scope array, sized for kNoAllocMaxT tokens and 256 local experts (the
// pick lists and chunk counts stay in the routing CTA's shared memory).  Every GPU that
// loads the library holds these bytes until the process exits, and every call on a device
// reuses the same bytes: calls that overlap on the GPU (two streams, or two host threads on
// one device) race on them and must be serialised by the caller.
constexpr int kNoAllocMaxT = 256;
constexpr size_t kNoAllocScratchBytes = 64 * 1024;
static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

struct NoAllocLayout {
  size_t plan, tok_nloc, tok_rows, tables, total;
};

__host__ __device__ constexpr size_t na_align(size_t x) { return (x + 255) / 256 * 256; }

__host__ __device__ constexpr NoAllocLayout noalloc_layout() {
  NoAllocLayout l{};
  l.plan = 0;
  l.tok_nloc = na_align(l.plan + sizeof(Plan));
  l.tok_rows = na_align(l.tok_nloc + kNoAllocMaxT * sizeof(int));
  l.tables = na_align(l.tok_rows + kNoAllocMaxT * kTopK * sizeof(int));
  l.total = na_align(l.tables + 3 * (kEG + 1) * sizeof(int));
  return l;
}
static_assert(noalloc_layout().total <= kNoAllocScratchBytes, "no-alloc scratch too small");

__global__ void __launch_bounds__(kRouteSmallThreads, 1) route_noalloc_kernel(RouteArgs a) {
  route_small_body<kNoAllocMaxT>(a);   // counts in shared memory: nothing carries over between calls
}

}  // namespace moe

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {};

}  // namespace

extern "C" MOE_B200_API int moe_b200_route_noalloc(const moe_b200_args* args, int32_t* topk_idx, float* topk_w,
                                                  int32_t* expert_count, int32_t* row_token, float* row_weight,
                                                  void* stream) {
  using namespace moe;
  if (!args) return report_error(MOE_B200_ERR_ARG, "null args");
  const int T = args->num_tokens, E = args->num_local_experts;
  if (T < 0 || E < 1 || E > kEG) return report_error(MOE_B200_ERR_ARG, "num_tokens < 0 or num_local_experts outside [1, 256]");
  if (T > kNoAllocMaxT)
    return report_error(MOE_B200_ERR_ARG,
                        "moe_b200_route_noalloc: num_tokens exceeds the static scratch limit of 256 tokens "
                        "(use moe_b200_route with a workspace)");
  if (T == 0) return MOE_B200_OK;
  if (!args->routing_logits || !args->routing_bias || !topk_idx || !topk_w || !expert_count || !row_token ||
      !row_weight)
    return report_error(MOE_B200_ERR_ARG, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(args->routing_logits) & 15u) != 0)
    return report_error(MOE_B200_ERR_ARG, "routing_logits must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return report_error(MOE_B200_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= 256) return report_error(MOE_B200_ERR_DEVICE, "device index out of range");
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return report_error(MOE_B200_ERR_DEVICE, "an sm_100 (B200-class) device is required");
  void* scratch = nullptr;
  {
    // one-time set-up per device (with that device current): the device address of the array.
    // The array's name in host code is only a host-side handle, never a device address.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_route_scratch);
      if (e != cudaSuccess) return report_error(MOE_B200_ERR_CUDA, cudaGetErrorString(e));
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  constexpr NoAllocLayout L = noalloc_layout();
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  RouteArgs r{};
  r.logits = args->routing_logits;
  r.bias = args->routing_bias;
  r.T = T;
  r.E = E;
  r.offset = args->local_expert_offset;
  r.rsf = args->routed_scaling_factor;
  r.nchunks = (T + kChunk - 1) / kChunk;
  r.r_pad = 0;
  r.plan = reinterpret_cast<Plan*>(sp + L.plan);
  r.topk_idx = topk_idx;
  r.topk_w = topk_w;
  r.tok_nloc = reinterpret_cast<int*>(sp + L.tok_nloc);
  r.tok_rows = reinterpret_cast<int*>(sp + L.tok_rows);   // pick lists and counts: shared memory
  int* tab = reinterpret_cast<int*>(sp + L.tables);
  r.e_count = expert_count;
  r.e_start = tab;
  r.e_mt_start = tab + (kEG + 1);
  r.e_tt = tab + 2 * (kEG + 1);
  r.row_token = row_token;
  r.row_weight = row_weight;
  // no activation copy and no output rows: routing and permutation metadata only
  r.hidden = nullptr;
  r.hs_scale = nullptr;
  r.out = nullptr;
  r.a_perm = nullptr;
  r.sa_perm = nullptr;
  route_noalloc_kernel<<<1, kRouteSmallThreads, 0, static_cast<cudaStream_t>(stream)>>>(r);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(MOE_B200_ERR_CUDA, cudaGetErrorString(e));
  return MOE_B200_OK;
}
