// Token-major grouped GEMMs for large T (prefill / expert-parallel batches), tcgen05 on
// sm_100a.  A tile is a block of routed token rows of one expert (MMA M = 128 rows) times
// 256 weight rows (MMA N = 256), so the tensor core runs at its full-width shape and every
// token row's fp32 scale is a per-thread scalar in the promotion.
//
//   MODE 1 (GEMM1): tile = (expert, 128-row token tile, pair tile nt: 128 X1 rows [128nt, +128)
//     and 128 X2 rows [2048+128nt, +128)); K = 56 blocks.  D = A . [W_X1 | W_X2]^T.
//       acc[r][c] += D[r][c] * sa[r, kb] * s13[e, block(c), kb]
//     epilogue: C = silu(X2) * X1, stored as the e4m3 pair C ~= s*(hi + lo), hi = e4m3(C/s),
//     lo = e4m3(C/s - hi), with one scale per (row, 128 columns), s = amax/448.
//   MODE 2 (GEMM2): tile = (expert, 128-token tile, 256 output features nt); K = 16 blocks.
//     hi and lo share every scale, so a K-block is one accumulation over the concatenation
//     [hi | lo]: four MMAs with A = hi, then four with A = lo, into the same accumulator.
//       acc[r][c] += D[r][c] * sc[token r, kb] * s2[e, nt, kb]
//     epilogue: a token with one local expert gets its bf16 output row directly, otherwise
//     w * O goes to its fp32 partial row, summed in ascending expert order by the combine
//     kernel (combine.cu).
//
// CTA = 12 warps: warp 2 TMA producer (one box per lane), warp 3 TMEM owner + single-thread MMA
// issuer (their warpgroup drops to 56 registers), warps 4..11 promotion/epilogue with 224
// registers: two warps per TMEM lane quarter, one per 128-column half of the accumulator.  The
// producer and the MMA issuer sit on the sub-partitions of lane quarters 2 and 3: the promotion
// warps of a quarter that shares its sub-partition with them read the accumulator late (their
// TMEM loads queue behind the issuers' instructions), and a partly filled token tile fills the
// quarters from 0 upward, so its live quarters are the undisturbed ones.
// Shared-memory stages: MODE 1 4 x 48 KB (128 token rows | 128 X1 rows | 128 X2 rows),
// MODE 2 3 x 64 KB (128 hi rows | 128 lo rows | 256 W2 rows); 2 TMEM accumulator buffers of 256
// columns.  Work: data-parallel
// whole tiles, then a stream-K tail (sched.cuh).  No TMA multicast (the kernels also run in the
// multi-GPU expert-parallel configuration).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "launch_args.cuh"
#include "moe_internal.cuh"
#include "ptx.cuh"
#include "sched.cuh"

namespace moe {

#ifdef MOE_TRACE
#define MOE_WCLK() clock64()
#define MOE_WADD(var, t0) (var) += clock64() - (t0)
// Per-K-block handoff timeline of CTA 0 (traced builds): `clock64` stamps in the trace region six
// kernel blocks past this kernel's counters (trace kernels 8 and 9), row-major [row][K-block]:
// row 0 MMA thread has a free accumulator, 1 its operand stage is full, 2 its MMAs and commits are
// issued, 3 the first promotion warp sees the accumulator, 4 + w promotion warp w releases it.
#define MOE_TL(g, row, n)                                                                          \
  do {                                                                                             \
    if (blockIdx.x == 0 && (n) < kTimelineKBs)                                                     \
      (g).trace[6 * kMaxSms * kTraceSlots + (row) * kTimelineKBs + (n)] = clock64();               \
  } while (0)
#else
#define MOE_WCLK() 0ll
#define MOE_WADD(var, t0) (void)0
#define MOE_TL(g, row, n) (void)0
#endif

template <int MODE>
struct WCfg;
template <>
struct WCfg<1> {
  static constexpr int KB = kKB1;
  static constexpr int NT = kNT1;     // 16 pair tiles
  static constexpr int STAGES = 4;
  static constexpr int STAGE_BYTES = 3 * 16384;
};
template <>
struct WCfg<2> {
  static constexpr int KB = kKB2;
  static constexpr int NT = kH / 256; // 28 feature tiles of 256
  static constexpr int STAGES = 3;
  static constexpr int STAGE_BYTES = 4 * 16384;
};
constexpr int kWRows = 128;      // token rows per tile (MMA M)
constexpr int kWProducerWarp = 2;   // sub-partition of lane quarter 2
constexpr int kWMmaWarp = 3;        // sub-partition of lane quarter 3; also owns the TMEM allocation

constexpr int kWThreads = 384;   // 3 warpgroups: producer/MMA (+2 idle warps), 2 x epilogue
constexpr int kWEpiThreads = 256;

template <int MODE>
struct WideSmem {
  uint8_t stage[WCfg<MODE>::STAGES][WCfg<MODE>::STAGE_BYTES];
  uint64_t full[WCfg<MODE>::STAGES];
  uint64_t empty[WCfg<MODE>::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int flag;
  float ssw[2][kKB1];      // this segment's weight scales (MODE 1: X1, X2 blocks)
  float amx[2][128];       // MODE 1: per-row amax of each column half
  int e_cnt[kEG + 1];
  int e_start[kEG + 1];
  int e_tiles[kEG + 1];
};

template <int MODE>
constexpr size_t wide_smem_bytes() {
  return sizeof(WideSmem<MODE>) + 1024;
}
static_assert(wide_smem_bytes<1>() <= 232448 && wide_smem_bytes<2>() <= 232448, "wide kernel shared memory");

struct WTile {
  int e, nt, row0, nr;
};

template <int MODE>
__device__ __forceinline__ WTile w_decode(const WideSmem<MODE>& sm, int E, int tile) {
  constexpr int NT = WCfg<MODE>::NT, ROWS = kWRows;
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sm.e_tiles[mid] * NT <= tile) lo = mid; else hi = mid - 1;
  }
  const int v = tile - sm.e_tiles[lo] * NT;
  const int jt = sm.e_tiles[lo + 1] - sm.e_tiles[lo];
  WTile s;
  s.e = lo;
  s.nt = v / jt;
  const int j = v - s.nt * jt;
  s.row0 = sm.e_start[lo] + ROWS * j;
  s.nr = min(ROWS, sm.e_cnt[lo] - ROWS * j);
  return s;
}

__device__ __forceinline__ float w_silu(float x) { return silu_fast(x); }

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// The whole producer warp runs this loop; each lane issues at most one box of a stage.  Tiled
// loads issued by one thread go through the TMA unit one after another (about 330 cycles per
// 16 KB box); issued by several lanes of a warp they overlap.
template <int MODE>
__device__ __forceinline__ void w_producer(WideSmem<MODE>& sm, const CUtensorMap* tmA, const CUtensorMap* tmA2,
                           const CUtensorMap* tmB, const TileArgs& g, const Sched& sk, int lane) {
  constexpr int ST = WCfg<MODE>::STAGES;
  uint32_t stage = 0, phase = 0, issued = 0, lastpar = 0;
  long long tw = 0, nkb = 0;
  // MODE 2: the first stages get their weight tiles before the dependency on GEMM1 resolves
  int pend_n = 0;
  int pend_row0[ST];
  int pend_kb[ST];
  bool waited = MODE == 1;
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  while (it.next(tile, k0, k1)) {
    const WTile s = w_decode<MODE>(sm, g.E, tile);
    for (int kb = k0; kb < k1; ++kb) {
      const long long t0 = MOE_WCLK();
      const bool ok = mbar_wait(&sm.empty[stage], phase ^ 1u, &sm.abort, g.status, kStWaitProducer);
      if (!__all_sync(0xffffffffu, ok)) goto drain;
      MOE_WADD(tw, t0);
      ++nkb;
      // the stage's byte count is armed before any lane's copy can complete it
      if (lane == 0) mbar_arrive_expect_tx(&sm.full[stage], WCfg<MODE>::STAGE_BYTES);
      __syncwarp();
      uint8_t* st = sm.stage[stage];
      if (MODE == 1) {
        if (lane == 0) tma_load_2d(st, tmA, &sm.full[stage], kb * kBlk, s.row0);
        if (lane == 1) tma_load_2d(st + 16384, tmB, &sm.full[stage], kb * kBlk, s.e * kN1 + s.nt * kBlk);
        if (lane == 2) tma_load_2d(st + 32768, tmB, &sm.full[stage], kb * kBlk, s.e * kN1 + kI + s.nt * kBlk);
      } else {
        if (lane == 2) tma_load_2d(st + 32768, tmB, &sm.full[stage], kb * kBlk, s.e * kH + s.nt * 256);
        if (lane == 3) tma_load_2d(st + 49152, tmB, &sm.full[stage], kb * kBlk, s.e * kH + s.nt * 256 + 128);
        if (!waited) {
          pend_row0[pend_n] = s.row0;
          pend_kb[pend_n] = kb;
          ++pend_n;
        } else if (lane < 2) {
          tma_load_2d(st + 16384 * lane, lane ? tmA2 : tmA, &sm.full[stage], kb * kBlk, s.row0);
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
            tma_load_2d(sm.stage[i] + 16384 * lane, lane ? tmA2 : tmA, &sm.full[i], pend_kb[i] * kBlk, pend_row0[i]);
        pend_n = 0;
      }
    }
  }
  if (MODE == 2 && !waited) {
    pdl_wait();
    for (int i = 0; i < pend_n; ++i)
      if (lane < 2)
        tma_load_2d(sm.stage[i] + 16384 * lane, lane ? tmA2 : tmA, &sm.full[i], pend_kb[i] * kBlk, pend_row0[i]);
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
__device__ __forceinline__ void w_mma(WideSmem<MODE>& sm, uint32_t tmem, const TileArgs& g, const Sched& sk) {
  constexpr int ST = WCfg<MODE>::STAGES;
  constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
  uint32_t stage = 0, phase = 0, tk = 0, buf = 0;
  int nkb = 0;
  long long tw_t = 0, tw_f = 0, t_first = 0, t_iss = 0;
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  while (it.next(tile, k0, k1)) {
    for (int kb = k0; kb < k1; ++kb) {
      long long t0 = MOE_WCLK();
      if (!mbar_wait(&sm.tempty[buf], ((tk >> buf) & 1u) ^ 1u, &sm.abort, g.status, kStWaitMmaTmem))
        goto done;
      MOE_TL(g, 0, nkb);
      MOE_WADD(tw_t, t0);
      t0 = MOE_WCLK();
      if (!mbar_wait(&sm.full[stage], phase, &sm.abort, g.status, kStWaitMma)) goto done;
      MOE_TL(g, 1, nkb);
      MOE_WADD(tw_f, t0);
#ifdef MOE_TRACE
      if (t_first == 0) t_first = static_cast<long long>(globaltimer_ns());
#endif
      tc_fence_after();
      t0 = MOE_WCLK();
      {
        const uint32_t st = smem_u32(sm.stage[stage]);
        const uint32_t d = tmem + buf * 256u;
        if (MODE == 1) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4(d, sdesc_k128_sw128(st + 32 * k), sdesc_k128_sw128(st + 16384 + 32 * k), idesc, k > 0);
        } else {
          // D = hi . W^T + lo . W^T over the K-block: A = hi, then A = lo, one accumulator
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_f8f6f4(d, sdesc_k128_sw128(st + 16384 * (k >> 2) + 32 * (k & 3)),
                       sdesc_k128_sw128(st + 32768 + 32 * (k & 3)), idesc, k > 0);
        }
      }
      mma_commit(&sm.empty[stage]);
      mma_commit(&sm.tfull[buf]);
      MOE_TL(g, 2, nkb);
      ++nkb;
      MOE_WADD(t_iss, t0);
      tk ^= 1u << buf;
      buf ^= 1u;
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
  g.trace[blockIdx.x * kTraceSlots + 14] = t_iss;
#endif
}

// MODE 1 tile epilogue: SwiGLU of this thread's 64 (X1, X2) column pairs of row `rit`, the row's
// 128-column amax (exchanged with the other column half), hi/lo e4m3 encoding and stores.
__device__ __forceinline__ void w_epi1(WideSmem<1>& sm, const TileArgs& g, const WTile& s, float* x1,
                                       const float* x2, int h, int rit, uint32_t* hw, uint32_t* lw) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 64; ++j) {
    x1[j] = w_silu(x2[j]) * x1[j];
    amax = fmaxf(amax, fabsf(x1[j]));
  }
  sm.amx[h][rit] = amax;
  named_bar_sync(1, kWEpiThreads);
  amax = fmaxf(sm.amx[0][rit], sm.amx[1][rit]);
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
#pragma unroll
  for (int j = 0; j < 64; j += 4) {
    const float y0 = x1[j] * inv, y1 = x1[j + 1] * inv, y2 = x1[j + 2] * inv, y3 = x1[j + 3] * inv;
    const uint32_t h01 = cvt_e4m3x2(y0, y1), h23 = cvt_e4m3x2(y2, y3);
    const float2 b01 = e4m3x2_to_f2(static_cast<uint16_t>(h01));
    const float2 b23 = e4m3x2_to_f2(static_cast<uint16_t>(h23));
    const uint32_t l01 = cvt_e4m3x2(y0 - b01.x, y1 - b01.y);
    const uint32_t l23 = cvt_e4m3x2(y2 - b23.x, y3 - b23.y);
    hw[j / 4] = h01 | (h23 << 16);
    lw[j / 4] = l01 | (l23 << 16);
  }
  if (h == 0 && rit < s.nr)
    g.c_scale[static_cast<size_t>(s.nt) * g.r_pad + s.row0 + rit] = amax > 0.f ? amax / 448.0f : 1.0f;
}

// Stores this thread's 64 hi bytes and 64 lo bytes of its row (columns 64h.. of the tile's 128)
// straight from registers: two 256-bit stores each, whole 32-byte sectors per lane.
__device__ __forceinline__ void w_store1(const TileArgs& g, const WTile& s, const uint32_t* hw, const uint32_t* lw,
                                         int h, int rit) {
  if (rit >= s.nr) return;
  const size_t off = static_cast<size_t>(s.row0 + rit) * kI + static_cast<size_t>(s.nt) * kBlk + 64 * h;
  st_global_v8_b32(g.c_hi + off, hw);
  st_global_v8_b32(g.c_hi + off + 32, hw + 8);
  st_global_v8_b32(g.c_lo + off, lw);
  st_global_v8_b32(g.c_lo + off + 32, lw + 8);
}

// MODE 2 tile epilogue: this thread's 128 output columns of its token row, stored straight from
// registers: the bf16 output row for a token with one local expert, otherwise the
// routing-weighted fp32 row for the combine kernel (combine.cu).  Each lane writes whole 32-byte
// sectors of its own row (256-bit stores; bf16 rows with 128-bit stores when the output map is
// only 16-byte aligned), so the epilogue uses no shared memory and no warp barriers while the
// next tile's operands stream into the stages.
__device__ __forceinline__ void w_epi2(const TileArgs& g, const WTile& s, const float* acc, int h, int rit, int t,
                                       float w, int kt) {
  if (rit >= s.nr) return;
  const int col0 = s.nt * 256 + 128 * h;
  if (kt == 1) {
    uint16_t* dst = out_row(g.out, t) + col0;
    if (g.out.al32) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = bf16x2_bits(__fmul_rn(acc[16 * i + 2 * j], w), __fmul_rn(acc[16 * i + 2 * j + 1], w));
        st_global_v8_b32(dst + 16 * i, v);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        uint4 v;
        v.x = bf16x2_bits(__fmul_rn(acc[8 * i], w), __fmul_rn(acc[8 * i + 1], w));
        v.y = bf16x2_bits(__fmul_rn(acc[8 * i + 2], w), __fmul_rn(acc[8 * i + 3], w));
        v.z = bf16x2_bits(__fmul_rn(acc[8 * i + 4], w), __fmul_rn(acc[8 * i + 5], w));
        v.w = bf16x2_bits(__fmul_rn(acc[8 * i + 6], w), __fmul_rn(acc[8 * i + 7], w));
        *reinterpret_cast<uint4*>(dst + 8 * i) = v;
      }
    }
  } else {
    float* dst = g.part2 + static_cast<size_t>(s.row0 + rit) * kH + col0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(acc[8 * i + j], w);
      st_global_v8(dst + 8 * i, v);
    }
  }
}

template <int MODE>
__device__ __forceinline__ void w_epilogue(WideSmem<MODE>& sm, uint32_t tmem, const TileArgs& g, const Sched& sk, int warp, int lane) {
  constexpr int KB = WCfg<MODE>::KB;
  const int ew = warp - 4;
  const int q = warp & 3;
  const int h = ew >> 2;
  const int rit = q * 32 + lane;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
  uint32_t tk = 0, buf = 0;
  int nkb = 0;
  bool dead = false;
  long long tw = 0, tp = 0, te = 0, tf = 0, ts = 0;
  if (MODE == 2) pdl_wait();   // the C scales and the combine inputs come from GEMM1
  SegIter it(sk, blockIdx.x);
  int tile, k0, k1;
  while (it.next(tile, k0, k1)) {
    const WTile s = w_decode<MODE>(sm, g.E, tile);
    long long t0 = MOE_WCLK();
    // this thread's token row
    const int trow = rit;
    const size_t srow = static_cast<size_t>(s.row0 + min(trow, s.nr - 1));
    // a lane quarter holding only padding rows skips its TMEM loads and FMAs
    const bool qlive = 32 * q < s.nr;
    // MODE 2: the token metadata of this thread's row, fetched while the K loop runs
    int meta_t = 0, meta_k = 0;
    float meta_w = 0.f;
    const bool meta_mine = MODE == 2 && trow < s.nr;
    if (meta_mine) {
      meta_t = __ldg(g.row_token + s.row0 + trow);
      meta_w = __ldg(g.row_weight + s.row0 + trow);
    }
    const float* swp1;
    const float* swp2;
    if (MODE == 1) {
      swp1 = g.sw + (static_cast<size_t>(s.e) * 32 + s.nt) * kKB1;
      swp2 = g.sw + (static_cast<size_t>(s.e) * 32 + kNT1 + s.nt) * kKB1;
    } else {
      swp1 = g.sw + (static_cast<size_t>(s.e) * kNT2 + 2 * s.nt) * kKB2;        // features [256nt, +128)
      swp2 = g.sw + (static_cast<size_t>(s.e) * kNT2 + 2 * s.nt + 1) * kKB2;    // features [256nt+128, +128)
    }
    if (ew == 0)
      for (int i = lane; i < k1 - k0; i += 32) {
        sm.ssw[0][i] = __ldg(swp1 + k0 + i);
        sm.ssw[1][i] = __ldg(swp2 + k0 + i);
      }
    // the row's token scales, four K-blocks ahead
    float pf0 = __ldg(g.sa + static_cast<size_t>(k0) * g.r_pad + srow);
    float pf1 = k0 + 1 < k1 ? __ldg(g.sa + static_cast<size_t>(k0 + 1) * g.r_pad + srow) : 0.f;
    float pf2 = k0 + 2 < k1 ? __ldg(g.sa + static_cast<size_t>(k0 + 2) * g.r_pad + srow) : 0.f;
    float pf3 = k0 + 3 < k1 ? __ldg(g.sa + static_cast<size_t>(k0 + 3) * g.r_pad + srow) : 0.f;
    named_bar_sync(1, kWEpiThreads);
    MOE_WADD(ts, t0);
    float acc1[MODE == 1 ? 64 : 128], acc2[MODE == 1 ? 64 : 1];
#pragma unroll
    for (int j = 0; j < (MODE == 1 ? 64 : 128); ++j) acc1[j] = 0.f;
#pragma unroll
    for (int j = 0; j < (MODE == 1 ? 64 : 1); ++j) acc2[j] = 0.f;
    // this segment's weight scales, each read one K-block ahead of its use
    float wa_n = sm.ssw[MODE == 1 ? 0 : h][0], wb_n = sm.ssw[MODE == 1 ? 1 : h][0];
    for (int kb = k0; kb < k1; ++kb) {
      const int ki = kb - k0;
      const float wa = wa_n, wb = wb_n;
      if (ki + 1 < k1 - k0) {
        wa_n = sm.ssw[MODE == 1 ? 0 : h][ki + 1];
        wb_n = sm.ssw[MODE == 1 ? 1 : h][ki + 1];
      }
      const float sa = pf0;
      pf0 = pf1;
      pf1 = pf2;
      pf2 = pf3;
      pf3 = kb + 4 < k1 ? __ldg(g.sa + static_cast<size_t>(kb + 4) * g.r_pad + srow) : 0.f;
      t0 = MOE_WCLK();
      if (!dead && !mbar_wait(&sm.tfull[buf], (tk >> buf) & 1u, &sm.abort, g.status, kStWaitEpilogue))
        dead = true;
      if (warp == 4 && lane == 0) MOE_TL(g, 3, nkb);
      MOE_WADD(tw, t0);
      t0 = MOE_WCLK();
      if (!dead && !qlive) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tempty[buf]);
        if (lane == 0) MOE_TL(g, warp, nkb);   // row 4 + (warp - 4)
      }
      if (!dead && qlive) {
        // Promotion in four steps of 2 x 16 columns (MODE 1: X1 and X2 columns 64h + 16s ..;
        // MODE 2: columns 128h + 32s ..).  Each step's TMEM load is issued before the previous
        // step's FMAs, so its latency hides behind them; the buffer goes back to the MMA as
        // soon as the last load has landed.
        tc_fence_after();
        const uint32_t base = lane_base + buf * 256u;
        const float fa = sa * wa, fb = sa * wb;
        const float2 fav = make_float2(fa, fa), fbv = make_float2(fb, fb);
        auto col_a = [&](int st) -> uint32_t {
          return MODE == 1 ? base + 64u * h + 16u * st : base + 128u * h + 32u * st;
        };
        auto col_b = [&](int st) -> uint32_t {
          return MODE == 1 ? base + 128u + 64u * h + 16u * st : base + 128u * h + 32u * st + 16u;
        };
        uint32_t ra[32], rb[32];
        tmem_ld16x2_issue(col_a(0), col_b(0), ra);
        tmem_wait_ld32(ra);
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          uint32_t* cur = (st & 1) ? rb : ra;
          uint32_t* nxt = (st & 1) ? ra : rb;
          if (st < 3) {
            tmem_ld16x2_issue(col_a(st + 1), col_b(st + 1), nxt);
          } else {   // every TMEM read of this buffer has completed
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.tempty[buf]);
            if (lane == 0) MOE_TL(g, warp, nkb);   // row 4 + (warp - 4)
          }
          float* acc_a;
          float* acc_b;
          if constexpr (MODE == 1) {
            acc_a = acc1 + 16 * st;
            acc_b = acc2 + 16 * st;
          } else {
            acc_a = acc1 + 32 * st;
            acc_b = acc1 + 32 * st + 16;
          }
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float2 a1 = make_float2(acc_a[j], acc_a[j + 1]);
            float2 a2 = make_float2(acc_b[j], acc_b[j + 1]);
            a1 = __ffma2_rn(make_float2(__uint_as_float(cur[j]), __uint_as_float(cur[j + 1])), fav, a1);
            a2 = __ffma2_rn(make_float2(__uint_as_float(cur[16 + j]), __uint_as_float(cur[17 + j])), fbv, a2);
            acc_a[j] = a1.x;
            acc_a[j + 1] = a1.y;
            acc_b[j] = a2.x;
            acc_b[j + 1] = a2.y;
          }
          if (st < 3) tmem_wait_ld32(nxt);
        }
      }
      MOE_WADD(tp, t0);
      ++nkb;
      if (MODE == 2 && ki == 0 && meta_mine) meta_k = __ldg(g.tok_nloc + meta_t);   // t arrived by now
      tk ^= 1u << buf;
      buf ^= 1u;
    }
    t0 = MOE_WCLK();
    if (!(k0 == 0 && k1 == KB)) {
      // stream-K fixup: publish this CTA's partial; the last contributor sums them in CTA order.
      // Slot layout [256 columns][128 rows] (MODE 1 columns: X1 0..127, X2 128..255).
      const int slot = sk.slot(blockIdx.x, tile);
      float* p = g.part + static_cast<size_t>(slot) * 256 * 128;
      if (MODE == 1) {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          p[(64 * h + j) * 128 + rit] = acc1[j];
          p[(128 + 64 * h + j) * 128 + rit] = acc2[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 128; ++j) p[(128 * h + j) * 128 + rit] = acc1[j];
      }
      named_bar_sync(1, kWEpiThreads);
      if (ew == 0 && lane == 0) {
        const int expect = sk.last_cta(tile) - sk.first_cta(tile) + 1;
        const int prev = atomic_add_acq_rel_gpu(g.tile_cnt + tile, 1);
        const int last = prev == expect - 1;
        if (last) g.tile_cnt[tile] = 0;
        sm.flag = last;
      }
      named_bar_sync(1, kWEpiThreads);
      const int last = sm.flag;
      named_bar_sync(1, kWEpiThreads);
      if (!last) {
        MOE_WADD(tf, t0);
        continue;
      }
#pragma unroll
      for (int j = 0; j < (MODE == 1 ? 64 : 128); ++j) acc1[j] = 0.f;
#pragma unroll
      for (int j = 0; j < (MODE == 1 ? 64 : 1); ++j) acc2[j] = 0.f;
      for (int cta = sk.first_cta(tile); cta <= sk.last_cta(tile); ++cta) {
        const float* pp = g.part + static_cast<size_t>(sk.slot(cta, tile)) * 256 * 128;
        if (MODE == 1) {
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            acc1[j] += __ldcg(pp + (64 * h + j) * 128 + rit);
            acc2[j] += __ldcg(pp + (128 + 64 * h + j) * 128 + rit);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 128; ++j) acc1[j] += __ldcg(pp + (128 * h + j) * 128 + rit);
        }
      }
    }
    MOE_WADD(tf, t0);
    t0 = MOE_WCLK();
    // (after an abort the epilogue still runs, on garbage, so every warp meets every barrier)
    if constexpr (MODE == 1) {
      uint32_t hw[16], lw[16];
      w_epi1(sm, g, s, acc1, acc2, h, rit, hw, lw);
      w_store1(g, s, hw, lw, h, rit);
    } else {
      w_epi2(g, s, acc1, h, rit, meta_t, meta_w, meta_k);
    }
    MOE_WADD(te, t0);
  }
#ifdef MOE_TRACE
  if (warp == 4 && lane == 0) {
    unsigned long long* tr = g.trace + blockIdx.x * kTraceSlots;
    tr[6] = tw;
    tr[7] = tp;
    tr[8] = te;
    tr[9] = tf;
    tr[10] = ts;
    tr[13] = clock64();
    tr[1] = globaltimer_ns();
  }
#endif
}

template <int MODE>
__global__ void __launch_bounds__(kWThreads, 1)
    wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmB, TileArgs g) {
  extern __shared__ uint8_t smem_raw[];
  WideSmem<MODE>& sm =
      *reinterpret_cast<WideSmem<MODE>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // GEMM1 waits for the routing; GEMM2 reads only the plan before its epilogue's wait.  Both let
  // their dependent kernel (GEMM2, the combine) launch at once.
  if (MODE == 1) pdl_wait();
  pdl_launch_dependents();
  const Plan plan = *g.plan;
  const int ntiles = plan.m_tiles * WCfg<MODE>::NT;
  Sched sk;
  sk.init(ntiles, gridDim.x, WCfg<MODE>::KB);
  if (ntiles == 0 || !sk.has_work(blockIdx.x)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i <= g.E; i += blockDim.x) {
    sm.e_cnt[i] = i < g.E ? g.e_count[i] : 0;
    sm.e_start[i] = g.e_start[i];
    sm.e_tiles[i] = g.e_tiles[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < WCfg<MODE>::STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.tfull[b], 1);
      mbar_init(&sm.tempty[b], 8);
    }
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmB);
  }
  if (warp == kWMmaWarp) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
#ifdef MOE_TRACE
  if (threadIdx.x == 0) {
    g.trace[blockIdx.x * kTraceSlots + 0] = globaltimer_ns();
    g.trace[blockIdx.x * kTraceSlots + 12] = clock64();
  }
#endif
  const uint32_t tmem = sm.tmem_base;
  // 384 threads x 168 registers at launch = 128 x 56 (producer/MMA warpgroup) + 256 x 224
  if (warp < 4) {
    setmaxnreg_dec<56>();
    if (warp == kWProducerWarp) {
      w_producer<MODE>(sm, &tmA, &tmA2, &tmB, g, sk, lane);
    } else if (warp == kWMmaWarp) {
      if (lane == 0) w_mma<MODE>(sm, tmem, g, sk);
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<224>();
    w_epilogue<MODE>(sm, tmem, g, sk, warp, lane);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

cudaError_t wide_prepare() {
  cudaError_t e = cudaFuncSetAttribute(wide_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(wide_smem_bytes<1>()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(wide_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(wide_smem_bytes<2>()));
}

// Launched as programmatic dependents of the preceding kernel in the stream (PDL).
cudaError_t wide_launch(int mode, int grid, cudaStream_t st, const CUtensorMap& a, const CUtensorMap& a2,
                        const CUtensorMap& b, const TileArgs& g) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (mode == 1) {
    cfg.dynamicSmemBytes = wide_smem_bytes<1>();
    return cudaLaunchKernelEx(&cfg, wide_kernel<1>, a, a2, b, g);
  }
  cfg.dynamicSmemBytes = wide_smem_bytes<2>();
  return cudaLaunchKernelEx(&cfg, wide_kernel<2>, a, a2, b, g);
}

}  // namespace moe
