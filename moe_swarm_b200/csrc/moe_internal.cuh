// Shared constants, the device-side plan and the workspace layout of one layer call.
#pragma once

#include <cstddef>
#include <cstdint>

namespace moe {

constexpr int kH = 7168;          // hidden size
constexpr int kI = 2048;          // intermediate size
constexpr int kN1 = 2 * kI;       // GEMM1 output rows per expert (X1 | X2)
constexpr int kEG = 256;          // global experts
constexpr int kTopK = 8;
constexpr int kNGroup = 8;
constexpr int kTopKGroup = 4;
constexpr int kBlk = 128;         // quantisation block edge
constexpr int kKB1 = kH / kBlk;   // 56 K-blocks of GEMM1
constexpr int kKB2 = kI / kBlk;   // 16 K-blocks of GEMM2
constexpr int kNT1 = kI / kBlk;   // 16 GEMM1 tiles (128 X1 + 128 X2 rows each)
constexpr int kNT2 = kH / kBlk;   // 56 GEMM2 tiles (128 output features each)

constexpr int kChunk = 128;       // tokens per rank-mask chunk of the permutation
constexpr int kRouteWarps = 8;    // routing / scatter CTAs: one token per warp
constexpr int kRouteThreads = kRouteWarps * 32;
constexpr int kCombineThreads = 256;                      // combine CTA: one float4 per thread
constexpr int kCombineChunks = kH / 4 / kCombineThreads;  // 7 row chunks per token
constexpr int kTok = 32;          // token tile (MMA N) of the streaming kernels
constexpr int kMaxSms = 256;      // partial-slot capacity of the stream-K fixup (2 per CTA)
constexpr int kStreamMaxT = 512;  // T above which the wide (token-major) kernels run
constexpr int kTraceSlots = 16;   // per-CTA counters of a traced build (MOE_TRACE)
constexpr int kTraceKernels = 10; // stream GEMM1, stream GEMM2, wide GEMM1, wide GEMM2, routing,
                                  // scatter, GEMM1 finalize, combine; then the per-K-block handoff
                                  // timelines of CTA 0 of wide GEMM1 and wide GEMM2
constexpr int kTimelineKBs = 256; // K-blocks recorded per timeline (rows of kTimelineKBs stamps)

// Bound of every device-side wait (mbarrier phases, stream-K arrivals, peer flags): far above
// any legitimate stall.  The peer-flag wait of expert parallelism takes a caller-given bound
// instead when one is passed (moe_b200_ep::wait_limit_us).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s

// Device status codes (first one wins).
enum : int {
  kStOk = 0,
  kStWaitProducer = 0x101,
  kStWaitMma = 0x102,
  kStWaitMmaTmem = 0x103,
  kStWaitEpilogue = 0x104,
  kStWaitDrain = 0x105,
  kStWaitFixup = 0x106,   // a split tile's finisher waiting for the other contributors
  kStWaitPeers = 0x107,   // expert parallelism: waiting for the other ranks' rows (ep.cu)
};

// Written by the routing scan, read by the GEMM kernels.
struct Plan {
  int T, E, rows;
  int m_tiles;            // 128-row token tiles (wide kernels)
  int tt;                 // 32-row token tiles (streaming kernels)
  int pad[3];
};

struct Layout {
  int T, E, nchunks;
  size_t r_max, r_pad, mt_max;
  // offsets in bytes
  size_t plan, route_done, status;
  size_t topk_idx, topk_w, tok_nloc, tok_le, tok_lw, tok_rows;
  size_t chunk_hist, chunk_base;
  size_t e_count, e_start, e_mt_start, e_tt;
  size_t sk_part, sk_cnt, trace;
  size_t row_token, row_weight, row_nloc;
  size_t a_perm, sa_perm;
  size_t c_hi, c_lo, c_scale;
  size_t part2;
  size_t counters_begin, counters_end;   // region zeroed by workspace_init
  size_t total;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline bool compute_layout(int T, int E, Layout* L) {
  if (T < 0 || E < 1 || E > kEG) return false;
  Layout l{};
  l.T = T;
  l.E = E;
  l.nchunks = (T + kChunk - 1) / kChunk;
  const size_t tt = T > 0 ? T : 1;
  const size_t per_tok = E < kTopK ? E : kTopK;
  l.r_max = tt * per_tok;
  l.r_pad = align_up(l.r_max, 32);
  l.mt_max = (l.r_max + kBlk - 1) / kBlk + E;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = align_up(o, 1024);
    o = at + bytes;
    return at;
  };
  l.plan = take(sizeof(Plan));
  // self-resetting counters and the status word live together so one memset clears them
  l.counters_begin = align_up(o, 1024);
  l.route_done = take(sizeof(int));
  l.status = take(sizeof(int));
  l.chunk_hist = take((size_t)(l.nchunks > 0 ? l.nchunks : 1) * E * sizeof(int));
  l.sk_cnt = take(((l.r_max + kTok - 1) / kTok + E) * kNT2 * sizeof(int));
  l.counters_end = align_up(o, 1024);
  l.topk_idx = take(tt * kTopK * sizeof(int));
  l.topk_w = take(tt * kTopK * sizeof(float));
  l.tok_nloc = take(tt * sizeof(int));
  l.tok_le = take(tt * kTopK * sizeof(int));
  l.tok_lw = take(tt * kTopK * sizeof(float));
  l.tok_rows = take(tt * kTopK * sizeof(int));
  l.chunk_base = take((size_t)(l.nchunks > 0 ? l.nchunks : 1) * E * sizeof(int));
  l.e_count = take((size_t)E * sizeof(int));
  l.e_start = take((size_t)(E + 1) * sizeof(int));
  l.e_mt_start = take((size_t)(E + 1) * sizeof(int));
  l.e_tt = take((size_t)(E + 1) * sizeof(int));
  l.row_token = take(l.r_pad * sizeof(int));
  l.row_weight = take(l.r_pad * sizeof(float));
  l.row_nloc = take(l.r_pad * sizeof(int));   // the row's token's local expert count
  l.a_perm = take(l.r_pad * kH);
  l.sa_perm = take((size_t)kKB1 * l.r_pad * sizeof(float));
  l.c_hi = take(l.r_pad * kI);
  l.c_lo = take(l.r_pad * kI);
  l.c_scale = take((size_t)kKB2 * l.r_pad * sizeof(float));
  l.part2 = take(l.r_pad * kH * sizeof(float));   // fp32 rows of tokens with > 1 local expert
  l.sk_part = take((size_t)2 * kMaxSms * 128 * 256 * sizeof(float));
  l.trace = take((size_t)kTraceKernels * kMaxSms * kTraceSlots * sizeof(unsigned long long));
  l.total = align_up(o, 1024);
  *L = l;
  return true;
}

}  // namespace moe
