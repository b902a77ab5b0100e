// Weight-streaming grouped GEMMs for small and mid T (decode regime), tcgen05 on sm_100a.
//
// Orientation is weight-major ("swap AB"): a tile is 128 weight rows (MMA M) times a
// 32-token tile of one expert (MMA N = 32), so an expert with a handful of routed tokens
// costs one N=32 MMA per 128x128 weight block and every weight byte is read from HBM once.
//
//   MODE 1 (GEMM1): tile = (expert, 32-token tile, pair tile nt of 128 X1 rows [128nt, +128)
//     and 128 X2 rows [2048+128nt, +128)); K = 56 blocks of 128.
//       D1 = W13[X1 rows] . A^T,  D2 = W13[X2 rows] . A^T   (fp8 x fp8 -> fp32 TMEM)
//       acc_i[r][c] += D_i[r][c] * s13[e, block_i, kb] * sa[token c, kb]   (exact fp32 scales)
//     The token tile A is gathered straight from hidden_states, four rows per TMA tile::gather4
//     (the routing writes only the permutation, no row copies), and sa is read at each token.
//     epilogue: C = silu(X2) * X1 per (feature r, token c); per-token amax over the tile's
//     128 features; C stored as the e4m3 pair C ~= s*(hi + lo), hi = e4m3(C/s),
//     lo = e4m3(C/s - hi), s = amax/448.  A tile that stream-K split over several CTAs is
//     summed and finished by stream_fin1_kernel, a programmatic dependent of this kernel, so
//     no CTA's range ends with a latency-bound fixup and epilogue on the critical path.
//   MODE 2 (GEMM2): tile = (expert, 32-token tile, 128 output features nt); K = 16 blocks.
//       D = W2 . [C_hi; C_lo]^T   (one N = 64 MMA: columns c and 32 + c are token c's hi and
//                                  lo products, which share every scale)
//       acc[r][c] += (D[r][c] + D[r][32 + c]) * s2[e, nt, kb] * sc[token c, kb]
//     epilogue: out[t, f] = bf16(w * O) for a token with one local expert; otherwise w * O
//     goes to the token's fp32 partial row, summed in ascending expert order by the combine
//     kernel (combine.cu) -- deterministic.  A split tile is finished by its first contributor,
//     which in stream-K order reaches it last and adds the others' partials in CTA order.
//
// Work is split stream-K over the persistent CTAs (sched.cuh), so all SMs stream weights
// even when routing activates a few experts.  CTA = 6 warps: warp 0 TMA producer, warp 1
// TMEM owner + single-thread MMA issuer, warps 2..5 promotion/epilogue (one per TMEM lane
// quarter; thread = weight row).  5 (MODE 1) / 8 (MODE 2) smem stages, 8 TMEM accumulator
// buffers of 64 columns, so the MMA runs up to 8 K-blocks ahead of the promotion.  No TMA
// multicast (the kernels also run in the multi-GPU expert-parallel configuration).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "launch_args.cuh"
#include "moe_internal.cuh"
#include "ptx.cuh"
#include "sched.cuh"

namespace moe {

// Per-CTA role counters of a traced build: [0] start ns, [1] end ns, [2] producer cycles
// waiting for a free stage, [3] K-blocks issued, [4] MMA cycles waiting for data, [5] MMA
// cycles waiting for a free TMEM buffer, [6] epilogue cycles waiting for an accumulator,
// [7] epilogue promotion cycles, [8] tile-epilogue cycles, [9] stream-K fixup cycles,
// [10] scale-staging cycles, [11] first data arrival ns, [12] MMA issue cycles (after the
// waits, through the commits), [13] MMA thread end ns.
#ifdef MOE_TRACE
#define MOE_TCLK() clock64()
#define MOE_TADD(var, t0) (var) += clock64() - (t0)
#else
#define MOE_TCLK() 0ll
#define MOE_TADD(var, t0) (void)0
#endif

template <int MODE>
struct SCfg;
template <>
struct SCfg<1> {
  static constexpr int KB = kKB1;
  static constexpr int NT = kNT1;
  static constexpr int STAGES = 5;
  static constexpr int STAGE_BYTES = 2 * 16384 + kTok * 128;   // W X1 | W X2 | tokens
};
template <>
struct SCfg<2> {
  static constexpr int KB = kKB2;
  static constexpr int NT = kNT2;
  static constexpr int STAGES = 8;
  static constexpr int STAGE_BYTES = 16384 + 2 * kTok * 128;   // W2 | C hi | C lo
};

constexpr int kSBufs = 8;          // TMEM accumulator buffers (64 columns each)
constexpr int kSThreads = 192;
constexpr int kSEpiThreads = 128;

template <int MODE>
struct StreamSmem {
  uint8_t stage[SCfg<MODE>::STAGES][SCfg<MODE>::STAGE_BYTES];
  uint8_t ostage[MODE == 1 ? 2 : 1][MODE == 1 ? kTok : 1][128];   // MODE 1: hi/lo bytes, [token][feature]
  float ssa[SCfg<MODE>::KB][kTok];   // this segment's token scales, [K-block][token column]
  float ssw[2][SCfg<MODE>::KB];      // this segment's weight scales (MODE 1: X1, X2 blocks)
  uint64_t full[SCfg<MODE>::STAGES];
  uint64_t empty[SCfg<MODE>::STAGES];
  uint64_t tfull[kSBufs];
  uint64_t tempty[kSBufs];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  // MODE 2 tile metadata, by segment parity: where token column c's output row goes -- its bf16
  // output row (bit 0 set) for a token with one local expert, else its fp32 partial row -- and
  // the row's combine weight.  The destination is resolved once per segment and column, not at
  // every store (the output map of expert parallelism divides and indexes per token).
  uintptr_t col_dst[2][kTok];
  float col_w[2][kTok];
  float colmax[4][kTok];
  float amax[kTok];
  int e_cnt[kEG + 1];
  int e_start[kEG + 1];
  int e_tt[kEG + 1];
};

template <int MODE>
constexpr size_t stream_smem_bytes() {
  return sizeof(StreamSmem<MODE>) + 1024;
}

struct STile {
  int e, nt, row0, nr;
};

template <int MODE, class SM>
__device__ __forceinline__ STile s_decode(const SM& sm, int E, int tile) {
  constexpr int NT = SCfg<MODE>::NT;
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sm.e_tt[mid] * NT <= tile) lo = mid; else hi = mid - 1;
  }
  const int v = tile - sm.e_tt[lo] * NT;
  const int jt = sm.e_tt[lo + 1] - sm.e_tt[lo];
  STile s;
  s.e = lo;
  s.nt = v / jt;
  const int j = v - s.nt * jt;
  s.row0 = sm.e_start[lo] + kTok * j;
  s.nr = min(kTok, sm.e_cnt[lo] - kTok * j);
  return s;
}

__device__ __forceinline__ float silu_f(float x) { return silu_fast(x); }

__device__ __forceinline__ uint16_t bf16_bits(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}

// The whole producer warp runs this loop; lane j issues box j of a stage, so a stage's boxes
// do not queue behind one another in the TMA unit as they do when one thread issues them all.
template <int MODE>
__device__ void s_producer(StreamSmem<MODE>& sm, const CUtensorMap* tmW, const CUtensorMap* tmT,
                           const CUtensorMap* tmT2, const TileArgs& g, const Sched& sk, int lane) {
  constexpr int ST = SCfg<MODE>::STAGES;
  uint32_t stage = 0, phase = 0, issued = 0, lastpar = 0;
  long long tw = 0, nkb = 0;
  // MODE 2: the first ST stages get their weight tiles before the dependency on GEMM1 is
  // resolved; their token tiles follow the wait.
  int pend_n = 0;
  int pend_row0[ST];
  int pend_kb[ST];
  bool waited = MODE == 1;
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  while (it.next(tile, k0, k1)) {
    const STile s = s_decode<MODE>(sm, g.E, tile);
    // MODE 1: lanes 2..9 gather the tile's 32 token rows from hidden_states, four per lane (rows
    // past the tile's tokens repeat its last token; their products are never stored)
    int tk0 = 0, tk1 = 0, tk2 = 0, tk3 = 0;
    if (MODE == 1 && lane >= 2 && lane < 2 + kTok / 4) {
      const int j = 4 * (lane - 2), last = s.row0 + s.nr - 1;
      tk0 = __ldg(g.row_token + min(s.row0 + j, last));
      tk1 = __ldg(g.row_token + min(s.row0 + j + 1, last));
      tk2 = __ldg(g.row_token + min(s.row0 + j + 2, last));
      tk3 = __ldg(g.row_token + min(s.row0 + j + 3, last));
    }
    for (int kb = k0; kb < k1; ++kb) {
      const long long t0 = MOE_TCLK();
      const bool ok = mbar_wait(&sm.empty[stage], phase ^ 1u, &sm.abort, g.status, kStWaitProducer);
      if (!__all_sync(0xffffffffu, ok)) goto drain;
      MOE_TADD(tw, t0);
      ++nkb;
      if (lane == 0) mbar_arrive_expect_tx(&sm.full[stage], SCfg<MODE>::STAGE_BYTES);
      __syncwarp();
      uint8_t* st = sm.stage[stage];
      if (MODE == 1) {
        if (lane == 0) tma_load_2d(st, tmW, &sm.full[stage], kb * kBlk, s.e * kN1 + s.nt * kBlk);
        if (lane == 1) tma_load_2d(st + 16384, tmW, &sm.full[stage], kb * kBlk, s.e * kN1 + kI + s.nt * kBlk);
        if (lane >= 2 && lane < 2 + kTok / 4)
          tma_gather4(st + 32768 + 512 * (lane - 2), tmT, &sm.full[stage], kb * kBlk, tk0, tk1, tk2, tk3);
      } else {
        if (lane == 2) tma_load_2d(st, tmW, &sm.full[stage], kb * kBlk, s.e * kH + s.nt * kBlk);
        if (!waited) {
          pend_row0[pend_n] = s.row0;
          pend_kb[pend_n] = kb;
          ++pend_n;
        } else if (lane < 2) {
          tma_load_2d(st + 16384 + lane * (kTok * 128), lane ? tmT2 : tmT, &sm.full[stage], kb * kBlk, s.row0);
        }
      }
      issued |= 1u << stage;
      lastpar = (lastpar & ~(1u << stage)) | (phase << stage);
      if (++stage == ST) {
        stage = 0;
        phase ^= 1u;
      }
      if (MODE == 2 && !waited && pend_n == ST) {
        pdl_wait();
        waited = true;
        for (int i = 0; i < pend_n; ++i)
          if (lane < 2)
            tma_load_2d(sm.stage[i] + 16384 + lane * (kTok * 128), lane ? tmT2 : tmT, &sm.full[i], pend_kb[i] * kBlk,
                        pend_row0[i]);
        pend_n = 0;
      }
    }
  }
  if (MODE == 2 && !waited) {   // fewer K-blocks than stages
    pdl_wait();
    for (int i = 0; i < pend_n; ++i)
      if (lane < 2)
        tma_load_2d(sm.stage[i] + 16384 + lane * (kTok * 128), lane ? tmT2 : tmT, &sm.full[i], pend_kb[i] * kBlk,
                    pend_row0[i]);
  }
drain:
  if (lane == 0)
    for (int s = 0; s < ST; ++s)
      if ((issued >> s) & 1u) {
        int no_abort = 0;
        mbar_wait(&sm.full[s], (lastpar >> s) & 1u, &no_abort, g.status, kStWaitDrain);
      }
  __syncwarp();
#ifdef MOE_TRACE
  if (lane == 0) {
    g.trace[blockIdx.x * kTraceSlots + 2] = tw;
    g.trace[blockIdx.x * kTraceSlots + 3] = nkb;
  }
#endif
}

template <int MODE>
__device__ void s_mma(StreamSmem<MODE>& sm, uint32_t tmem, const TileArgs& g, const Sched& sk) {
  constexpr int ST = SCfg<MODE>::STAGES;
  constexpr uint32_t idesc = idesc_e4m3_f32(128, kTok);
  constexpr uint32_t idesc_hilo = idesc_e4m3_f32(128, 2 * kTok);   // MODE 2: B = [C_hi; C_lo]
  uint32_t stage = 0, phase = 0, tk = 0, buf = 0;
  long long tw_t = 0, tw_f = 0, t_first = 0, t_iss = 0;
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  while (it.next(tile, k0, k1)) {
    for (int kb = k0; kb < k1; ++kb) {
      long long t0 = MOE_TCLK();
      if (!mbar_wait(&sm.tempty[buf], ((tk >> buf) & 1u) ^ 1u, &sm.abort, g.status, kStWaitMmaTmem))
        goto done;
      MOE_TADD(tw_t, t0);
      t0 = MOE_TCLK();
      if (!mbar_wait(&sm.full[stage], phase, &sm.abort, g.status, kStWaitMma)) goto done;
      MOE_TADD(tw_f, t0);
#ifdef MOE_TRACE
      if (t_first == 0) t_first = static_cast<long long>(globaltimer_ns());
#endif
      tc_fence_after();
      t0 = MOE_TCLK();
      {
        const uint32_t st = smem_u32(sm.stage[stage]);
        const uint32_t d = tmem + buf * 64u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (MODE == 1) {
            const uint64_t bt = sdesc_k128_sw128(st + 32768 + 32 * k);
            mma_f8f6f4(d, sdesc_k128_sw128(st + 32 * k), bt, idesc, k > 0);
            mma_f8f6f4(d + 32u, sdesc_k128_sw128(st + 16384 + 32 * k), bt, idesc, k > 0);
          } else {
            // the hi and lo token tiles lie back to back in the stage (same 128-byte swizzle,
            // 1024-byte aligned), so together they are one 64-row B operand: one N = 64 MMA
            // gives W2.C_hi in columns 0..31 and W2.C_lo in 32..63, reading W2 once
            mma_f8f6f4(d, sdesc_k128_sw128(st + 32 * k), sdesc_k128_sw128(st + 16384 + 32 * k), idesc_hilo, k > 0);
          }
        }
      }
      mma_commit(&sm.empty[stage]);
      mma_commit(&sm.tfull[buf]);
      MOE_TADD(t_iss, t0);
      tk ^= 1u << buf;
      buf = (buf + 1) & (kSBufs - 1);
      if (++stage == ST) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
done:
  mma_commit(&sm.drain);
  int no_abort = 0;
  mbar_wait(&sm.drain, 0, &no_abort, g.status, kStWaitDrain);
#ifdef MOE_TRACE
  g.trace[blockIdx.x * kTraceSlots + 4] = tw_f;
  g.trace[blockIdx.x * kTraceSlots + 5] = tw_t;
  g.trace[blockIdx.x * kTraceSlots + 11] = t_first;
  g.trace[blockIdx.x * kTraceSlots + 12] = t_iss;
  g.trace[blockIdx.x * kTraceSlots + 13] = globaltimer_ns();
#endif
}

// MODE 1 tile epilogue: SwiGLU, per-token amax over the 128 features, hi/lo e4m3 encoding.
template <class SM>
__device__ void s_epi1(SM& sm, const TileArgs& g, const STile& s, float* x1, const float* x2, int q, int lane) {
  const int r = q * 32 + lane;
  float m[kTok];
#pragma unroll
  for (int c = 0; c < kTok; ++c) {
    const float v = silu_f(x2[c]) * x1[c];
    x1[c] = v;
    m[c] = fabsf(v);
  }
  warp_colmax32(m, lane);
  sm.colmax[q][lane] = m[0];
  named_bar_sync(1, kSEpiThreads);
  if (q == 0) {
    const float a = fmaxf(fmaxf(sm.colmax[0][lane], sm.colmax[1][lane]), fmaxf(sm.colmax[2][lane], sm.colmax[3][lane]));
    sm.amax[lane] = a;
    if (lane < s.nr)
      g.c_scale[static_cast<size_t>(s.nt) * g.r_pad + s.row0 + lane] = a > 0.f ? a / 448.0f : 1.0f;
  }
  named_bar_sync(1, kSEpiThreads);
#pragma unroll
  for (int c = 0; c < kTok; c += 2) {
    const float a0 = sm.amax[c], a1 = sm.amax[c + 1];
    const float y0 = x1[c] * (a0 > 0.f ? 448.0f / a0 : 0.f);
    const float y1 = x1[c + 1] * (a1 > 0.f ? 448.0f / a1 : 0.f);
    const uint32_t h = cvt_e4m3x2(y0, y1);
    const float2 b = e4m3x2_to_f2(static_cast<uint16_t>(h));
    const uint32_t l = cvt_e4m3x2(y0 - b.x, y1 - b.y);
    sm.ostage[0][c][r] = static_cast<uint8_t>(h & 0xFF);
    sm.ostage[0][c + 1][r] = static_cast<uint8_t>(h >> 8);
    sm.ostage[1][c][r] = static_cast<uint8_t>(l & 0xFF);
    sm.ostage[1][c + 1][r] = static_cast<uint8_t>(l >> 8);
  }
  named_bar_sync(1, kSEpiThreads);
  const int tid = q * 32 + lane;
  for (int i = tid; i < 2 * kTok * 8; i += kSEpiThreads) {
    const int h = i / (kTok * 8), c = (i / 8) % kTok, ch = i % 8;
    if (c < s.nr) {
      uint8_t* dst = (h == 0 ? g.c_hi : g.c_lo) + static_cast<size_t>(s.row0 + c) * kI + s.nt * kBlk + ch * 16;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&sm.ostage[h][c][ch * 16]);
    }
  }
  named_bar_sync(1, kSEpiThreads);
}

// MODE 2 tile epilogue: for each token column, the bf16 output row directly when the token
// has one local expert, otherwise the routing-weighted fp32 row for the combine kernel.
// The metadata was staged with the segment's scales (col_*[par]).
__device__ void s_epi2(StreamSmem<2>& sm, const TileArgs& g, const STile& s, const float* acc, int q,
                       int lane, int par) {
  const int r = q * 32 + lane;
  const int f = s.nt * kBlk + r;
#pragma unroll
  for (int c = 0; c < kTok; ++c) {
    if (c >= s.nr) break;
    const float v = __fmul_rn(acc[c], sm.col_w[par][c]);
    const uintptr_t d = sm.col_dst[par][c];
    if (d & 1u)
      reinterpret_cast<uint16_t*>(d & ~uintptr_t(1))[f] = bf16_bits(v);
    else
      reinterpret_cast<float*>(d)[f] = v;
  }
}

template <int MODE>
__device__ void s_epilogue(StreamSmem<MODE>& sm, uint32_t tmem, const TileArgs& g, const Sched& sk,
                           int warp, int lane) {
  const int q = warp & 3;
  const int r = q * 32 + lane;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
  uint32_t tk = 0, buf = 0;
  bool dead = false;
  long long tw = 0, tp = 0, te = 0, tf = 0, ts = 0;
  if (MODE == 2) pdl_wait();   // the C scales and the combine inputs come from GEMM1
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  int par = 1;   // segment parity (the double-buffered tile metadata)
  while (it.next(tile, k0, k1)) {
    par ^= 1;
    const STile s = s_decode<MODE>(sm, g.E, tile);
    long long t0 = MOE_TCLK();
    // lane c prefetches the scale of token column c (clamped to a routed row of this tile)
    const size_t srow = static_cast<size_t>(s.row0 + min(lane, s.nr - 1));
    float acc1[kTok], acc2[kTok];
#pragma unroll
    for (int c = 0; c < kTok; ++c) {
      acc1[c] = 0.f;
      acc2[c] = 0.f;
    }
    const float* swp1;
    const float* swp2;
    if (MODE == 1) {
      swp1 = g.sw + (static_cast<size_t>(s.e) * 32 + s.nt) * kKB1;
      swp2 = g.sw + (static_cast<size_t>(s.e) * 32 + kNT1 + s.nt) * kKB1;
    } else {
      swp1 = g.sw + (static_cast<size_t>(s.e) * kNT2 + s.nt) * kKB2;
      swp2 = swp1;
    }
    // stage the segment's scales in shared memory: one round of independent loads per
    // segment instead of an L2 round trip on every K-block's critical path
    const size_t scol = MODE == 1 && g.sa_by_token ? static_cast<size_t>(__ldg(g.row_token + srow)) : srow;
    for (int i = q; i < k1 - k0; i += 4) sm.ssa[i][lane] = __ldg(g.sa + static_cast<size_t>(k0 + i) * g.sa_ld + scol);
    if (q == 0)
      for (int i = lane; i < k1 - k0; i += 32) {
        sm.ssw[0][i] = __ldg(swp1 + k0 + i);
        sm.ssw[1][i] = __ldg(swp2 + k0 + i);
      }
    // MODE 2: the tile epilogue's metadata, in the same round of loads (lane c: token column c).
    // Double-buffered by segment parity: warps may still read the previous segment's copy.
    if (MODE == 2 && q == 1) {
      const bool live = lane < s.nr;
      const int t = live ? __ldg(g.row_token + s.row0 + lane) : 0;
      const int k = live ? __ldg(g.row_nloc + s.row0 + lane) : 0;
      sm.col_w[par][lane] = live ? __ldg(g.row_weight + s.row0 + lane) : 0.f;
      sm.col_dst[par][lane] = k == 1 ? reinterpret_cast<uintptr_t>(out_row(g.out, t)) | 1u
                                     : reinterpret_cast<uintptr_t>(g.part2 + static_cast<size_t>(s.row0 + lane) * kH);
    }
    named_bar_sync(1, kSEpiThreads);
    MOE_TADD(ts, t0);
    for (int kb = k0; kb < k1; ++kb) {
      const int ki = kb - k0;
      const float w1 = sm.ssw[0][ki], w2 = sm.ssw[1][ki];
      t0 = MOE_TCLK();
      if (!dead && !mbar_wait(&sm.tfull[buf], (tk >> buf) & 1u, &sm.abort, g.status, kStWaitEpilogue))
        dead = true;
      MOE_TADD(tw, t0);
      t0 = MOE_TCLK();
      if (!dead) {
        tc_fence_after();
        float d1[kTok], d2[kTok];
        tmem_ld32x2_wait(lane_base + buf * 64u, lane_base + buf * 64u + 32u, d1, d2);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tempty[buf]);
        const float4* sv = reinterpret_cast<const float4*>(sm.ssa[ki]);
#pragma unroll
        for (int c = 0; c < kTok; ++c) {
          const float4 s4 = sv[c / 4];
          const float sc = (c & 3) == 0 ? s4.x : (c & 3) == 1 ? s4.y : (c & 3) == 2 ? s4.z : s4.w;
          if (MODE == 1) {
            acc1[c] = fmaf(d1[c], sc * w1, acc1[c]);
            acc2[c] = fmaf(d2[c], sc * w2, acc2[c]);
          } else {
            acc1[c] = fmaf(d1[c] + d2[c], sc * w1, acc1[c]);   // hi and lo share every scale
          }
        }
      }
      MOE_TADD(tp, t0);
      tk ^= 1u << buf;
      buf = (buf + 1) & (kSBufs - 1);
    }
    t0 = MOE_TCLK();
    const bool full = (k0 == 0 && k1 == SCfg<MODE>::KB);
    if (!full) {
      // A split tile.  In stream-K order its first contributor (k0 == 0) reaches its segment at
      // the end of its range, the others earlier, so the first contributor finishes the tile:
      // the others store their partial (live token columns only) and signal one arrival without
      // waiting for anything; the finisher waits for those arrivals (normally all in already)
      // and adds their partials to its own in CTA order.  GEMM1's split tiles are all finished
      // by stream_fin1_kernel after this kernel instead, so there every contributor stores.
      constexpr int NH = MODE == 1 ? 2 : 1;
      const bool finisher = MODE == 2 && k0 == 0;
      if (!finisher) {
        const int slot = sk.slot(blockIdx.x, tile);
        float* p = g.part + static_cast<size_t>(slot) * NH * kTok * 128;
#pragma unroll
        for (int c = 0; c < kTok; ++c) {
          if (c >= s.nr) break;
          p[c * 128 + r] = acc1[c];
          if (MODE == 1) p[(kTok + c) * 128 + r] = acc2[c];
        }
        if (MODE == 2) {
          named_bar_sync(1, kSEpiThreads);   // the four warps' stores, then one release
          if (q == 0 && lane == 0) red_add_release_gpu(g.tile_cnt + tile, 1);
        }
        MOE_TADD(tf, t0);
        continue;
      }
      const int c0 = static_cast<int>(blockIdx.x), c1 = sk.last_cta(tile);
      if (q == 0 && lane == 0) {
        if (counter_wait_geq(g.tile_cnt + tile, c1 - c0, &sm.abort, g.status, kStWaitFixup))
          g.tile_cnt[tile] = 0;   // every other contributor has arrived: reset for the next call
      }
      named_bar_sync(1, kSEpiThreads);
      // live columns in blocks of 8; the loads of up to four contributors go out together
#pragma unroll
      for (int cb = 0; cb < kTok; cb += 8) {
        if (cb >= s.nr) break;
        for (int cta = c0 + 1; cta <= c1; cta += 4) {
          float v[4][8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (cta + j > c1) break;
            const float* pp = g.part + static_cast<size_t>(sk.slot(cta + j, tile)) * NH * kTok * 128 + cb * 128 + r;
#pragma unroll
            for (int c = 0; c < 8; ++c) v[j][c] = __ldcg(pp + c * 128);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (cta + j > c1) break;
#pragma unroll
            for (int c = 0; c < 8; ++c) acc1[cb + c] += v[j][c];
          }
        }
      }
    }
    MOE_TADD(tf, t0);
    t0 = MOE_TCLK();
    // (after an abort the epilogue still runs, on garbage, so every warp meets every barrier)
    if (MODE == 1)
      s_epi1(reinterpret_cast<StreamSmem<1>&>(sm), g, s, acc1, acc2, q, lane);
    else
      s_epi2(reinterpret_cast<StreamSmem<2>&>(sm), g, s, acc1, q, lane, par);
    MOE_TADD(te, t0);
  }
#ifdef MOE_TRACE
  if (warp == 2 && lane == 0) {
    unsigned long long* tr = g.trace + blockIdx.x * kTraceSlots;
    tr[6] = tw;
    tr[7] = tp;
    tr[8] = te;
    tr[9] = tf;
    tr[10] = ts;
    tr[1] = globaltimer_ns();
  }
#endif
}

template <int MODE>
__global__ void __launch_bounds__(kSThreads, 1)
    stream_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmT,
                  const __grid_constant__ CUtensorMap tmT2, TileArgs g) {
  extern __shared__ uint8_t smem_raw[];
  StreamSmem<MODE>& sm =
      *reinterpret_cast<StreamSmem<MODE>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // The barriers, the tensor-map prefetches and the TMEM allocation depend on no earlier kernel:
  // they run before the dependency wait.  GEMM1 depends on the routing kernel for everything
  // else; GEMM2 reads only the plan (routing, complete once GEMM1 started) before its own wait,
  // so it can prefetch weights while GEMM1 and the finalize end.  Both let their dependent
  // kernel launch at once, so its CTAs are resident and waiting when this grid ends.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < SCfg<MODE>::STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(&sm.tfull[b], 1);
      mbar_init(&sm.tempty[b], 4);
    }
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmT);
    tma_prefetch_desc(&tmT2);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  if (MODE == 1) pdl_wait();
  pdl_launch_dependents();
  const Plan plan = *g.plan;
  Sched sk;
  sk.init(plan.tt * SCfg<MODE>::NT, gridDim.x, SCfg<MODE>::KB);
  const bool work = plan.tt != 0 && sk.has_work(blockIdx.x);
  if (work)
    for (int i = threadIdx.x; i <= g.E; i += blockDim.x) {
      sm.e_cnt[i] = i < g.E ? g.e_count[i] : 0;
      sm.e_start[i] = g.e_start[i];
      sm.e_tt[i] = g.e_tiles[i];
    }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (!work) {   // no work for this CTA
    if (warp == 1) tmem_dealloc(sm.tmem_base, 512);
    return;
  }
#ifdef MOE_TRACE
  if (threadIdx.x == 0) g.trace[blockIdx.x * kTraceSlots + 0] = globaltimer_ns();
#endif
  const uint32_t tmem = sm.tmem_base;
  if (warp == 0) {
    s_producer<MODE>(sm, &tmW, &tmT, &tmT2, g, sk, lane);
  } else if (warp == 1) {
    if (lane == 0) s_mma<MODE>(sm, tmem, g, sk);
    __syncwarp();
  } else {
    s_epilogue<MODE>(sm, tmem, g, sk, warp, lane);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

cudaError_t stream_prepare() {
  cudaError_t e = cudaFuncSetAttribute(stream_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(stream_smem_bytes<1>()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(stream_smem_bytes<2>()));
}

// The plan read through L2 only (it may have been written by another grid after this SM cached it).
__device__ __forceinline__ Plan ld_cg_plan(const Plan* p) {
  const int4* q = reinterpret_cast<const int4*>(p);
  const int4 a = __ldcg(q), b = __ldcg(q + 1);
  Plan r;
  r.T = a.x;
  r.E = a.y;
  r.rows = a.z;
  r.m_tiles = a.w;
  r.tt = b.x;
  r.pad[0] = b.y;
  r.pad[1] = b.z;
  r.pad[2] = b.w;
  return r;
}

// Shared memory of stream_fin1_kernel: the tile tables.
struct FinSmem {
  int e_cnt[kEG + 1];
  int e_start[kEG + 1];
  int e_tt[kEG + 1];
};
constexpr int kFinThreads = 256;

// GEMM1 tiles that stream-K split over several CTAs, finished one (tile, token column) pair per
// warp: the contributors' partial accumulators summed in CTA order (deterministic; the same sums
// in the same order as a last-arriver fixup), then the column's SwiGLU, its amax over the tile's
// 128 features (a warp reduction) and its hi/lo e4m3 bytes -- element for element the arithmetic
// of s_epi1.  Lane l owns features 4l..4l+3: one float4 of X1 and one of X2 per contributor, and
// one 4-byte store each of the column's hi and lo bytes, so a column is one round of loads and
// two coalesced 128-byte stores with no block barrier.  Pairs are numbered column-major
// (p = column * nsplit + split tile), so at decode sizes, where a tile holds one or two tokens,
// the live pairs fall on distinct warps.  G is the GEMM's grid, which fixes its tile split.
__global__ void __launch_bounds__(kFinThreads) stream_fin1_kernel(TileArgs g, int G) {
  __shared__ FinSmem sm;
  MOE_TRACE_CTA(g.trace, 0);
  pdl_launch_dependents();    // GEMM2 may start its prologue and weight prefetch
  // The plan and the tile tables come from the routing, which completed before GEMM1 passed its
  // own dependency wait (and so before this grid was launched): they are read before this grid's
  // wait, from L2, while GEMM1 still runs.
  const Plan plan = ld_cg_plan(g.plan);
  for (int i = threadIdx.x; i <= g.E; i += blockDim.x) {
    sm.e_cnt[i] = i < g.E ? __ldcg(g.e_count + i) : 0;
    sm.e_start[i] = __ldcg(g.e_start + i);
    sm.e_tt[i] = __ldcg(g.e_tiles + i);
  }
  pdl_wait();                 // the partials come from GEMM1
  MOE_TRACE_CTA(g.trace, 2);
  Sched sk;
  sk.init(plan.tt * SCfg<1>::NT, G, SCfg<1>::KB);
  const int nsplit = sk.tiles - sk.dp;   // stream-K tiles
  __syncthreads();
  const int lane = threadIdx.x & 31;
  constexpr int kWarps = kFinThreads / 32;
  const int nwarps = static_cast<int>(gridDim.x) * kWarps;
  for (int p = static_cast<int>(blockIdx.x) * kWarps + (threadIdx.x >> 5); p < nsplit * kTok; p += nwarps) {
    const int c = p / nsplit;
    const int tile = sk.dp + (p - c * nsplit);
    const int c0 = sk.first_cta(tile), c1 = sk.last_cta(tile);
    if (c0 == c1) continue;   // one contributor: the GEMM finished this tile itself
    const STile s = s_decode<1>(sm, g.E, tile);
    if (c >= s.nr) continue;  // no token in this column
    float4 x1 = make_float4(0.f, 0.f, 0.f, 0.f), x2 = x1;
    for (int cta = c0; cta <= c1; cta += 4) {
      float4 v1[4], v2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (cta + j > c1) break;
        const float* pp = g.part + static_cast<size_t>(sk.slot(cta + j, tile)) * 2 * kTok * 128 + c * 128 + 4 * lane;
        v1[j] = __ldcg(reinterpret_cast<const float4*>(pp));
        v2[j] = __ldcg(reinterpret_cast<const float4*>(pp + kTok * 128));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (cta + j > c1) break;
        x1.x += v1[j].x;
        x1.y += v1[j].y;
        x1.z += v1[j].z;
        x1.w += v1[j].w;
        x2.x += v2[j].x;
        x2.y += v2[j].y;
        x2.z += v2[j].z;
        x2.w += v2[j].w;
      }
    }
    const float v0 = silu_f(x2.x) * x1.x, v1 = silu_f(x2.y) * x1.y;
    const float v2 = silu_f(x2.z) * x1.z, v3 = silu_f(x2.w) * x1.w;
    float m = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) g.c_scale[static_cast<size_t>(s.nt) * g.r_pad + s.row0 + c] = m > 0.f ? m / 448.0f : 1.0f;
    const float inv = m > 0.f ? 448.0f / m : 0.f;
    const float y0 = v0 * inv, y1 = v1 * inv, y2 = v2 * inv, y3 = v3 * inv;
    const uint32_t h01 = cvt_e4m3x2(y0, y1) & 0xFFFFu, h23 = cvt_e4m3x2(y2, y3) & 0xFFFFu;
    const float2 b01 = e4m3x2_to_f2(static_cast<uint16_t>(h01));
    const float2 b23 = e4m3x2_to_f2(static_cast<uint16_t>(h23));
    const uint32_t l01 = cvt_e4m3x2(y0 - b01.x, y1 - b01.y) & 0xFFFFu;
    const uint32_t l23 = cvt_e4m3x2(y2 - b23.x, y3 - b23.y) & 0xFFFFu;
    const size_t off = static_cast<size_t>(s.row0 + c) * kI + s.nt * kBlk + 4 * lane;
    *reinterpret_cast<uint32_t*>(g.c_hi + off) = h01 | (h23 << 16);
    *reinterpret_cast<uint32_t*>(g.c_lo + off) = l01 | (l23 << 16);
  }
  MOE_TRACE_CTA(g.trace, 1);
}

// Launched as a programmatic dependent of GEMM1.
// Four CTAs per GEMM CTA: a warp finishes its (tile, column) pairs one after another, each a chain
// of dependent loads, so more warps than pairs keep that chain to one round.
cudaError_t stream_fin_launch(int G, cudaStream_t st, const TileArgs& g) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(4 * G);
  cfg.blockDim = dim3(kFinThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, stream_fin1_kernel, g, G);
}

cudaError_t stream_launch(int mode, int grid, cudaStream_t st, const CUtensorMap& w, const CUtensorMap& t,
                          const CUtensorMap& t2, const TileArgs& g) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (mode == 1) {
    cfg.dynamicSmemBytes = stream_smem_bytes<1>();
    return cudaLaunchKernelEx(&cfg, stream_kernel<1>, w, t, t2, g);
  }
  cfg.dynamicSmemBytes = stream_smem_bytes<2>();
  return cudaLaunchKernelEx(&cfg, stream_kernel<2>, w, t, t2, g);
}

}  // namespace moe
