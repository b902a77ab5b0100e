// Kernel argument structs and launch constants shared by the kernels and the C-ABI launcher.
#pragma once

#include <cstddef>
#include <cstdint>

#include "moe_internal.cuh"

namespace moe {

// Where token t's bf16 output row goes: the caller's output (shard == 0), or -- expert
// parallelism over peer memory -- the receive buffer of the rank that owns t (owner t / shard),
// at this rank's slot, so the row crosses NVLink from the epilogue that produces it.
constexpr int kMaxRanks = 8;
struct OutMap {
  uint16_t* base[kMaxRanks];   // [0]: the output; EP: each rank's receive buffer (this call's phase)
  int shard;                   // tokens per rank; 0: a single output
  int slot_rows;               // EP: this rank's slot, rank * shard rows into each receive buffer
  int al32;                    // every base is 32-byte aligned (rows then are too: 14,336-byte pitch)
};

__host__ __device__ __forceinline__ uint16_t* out_row(const OutMap& m, int t) {
  if (m.shard == 0) return m.base[0] + static_cast<size_t>(t) * kH;
  const int r = t / m.shard;
  return m.base[r] + (static_cast<size_t>(m.slot_rows) + (t - r * m.shard)) * kH;
}

// The end of an expert-parallel call over peer memory (ep.cu).
struct EpArgs {
  unsigned int* signal[kMaxRanks];   // per rank: its flag words [2][kMaxRanks] (peer-mapped)
  const uint16_t* recv;              // this rank's receive buffer, this call's phase: [N][shard][kH]
  uint16_t* out;                     // this rank's shard [shard][kH]
  int world, rank, shard, phase;
  unsigned int epoch;
  unsigned long long wait_ns;        // bound of the wait for the peers' flags
  int* status;
};

struct RouteArgs {
  const float* logits;
  const uint16_t* bias;
  const uint8_t* hidden;
  const float* hs_scale;
  uint16_t* out;
  int T, E, offset;
  float rsf;
  // pre-routed calls (moe_b200_forward_routed): the caller's picks replace the routing
  const int* pre_idx;     // [T, 8] global expert ids, null for routed calls
  const float* pre_w;     // [T, 8] combine weights
  int nchunks;
  size_t r_pad;
  Plan* plan;
  int* route_done;
  int* topk_idx;
  float* topk_w;
  int* tok_nloc;
  int* tok_le;
  float* tok_lw;
  int* tok_rows;
  int* chunk_hist;
  int* chunk_base;
  int* e_count;
  int* e_start;
  int* e_mt_start;
  int* e_tt;
  int* row_token;
  float* row_weight;
  int* row_nloc;     // per row: its token's local expert count (null: not recorded)
  uint8_t* a_perm;
  float* sa_perm;
  unsigned long long* trace;   // [2][kMaxSms][kTraceSlots]: routing, scatter (MOE_TRACE builds)
};


// Start / end time of a CTA in a traced build (MOE_TRACE): slots [0] and [1] of the CTA's
// record, CTAs beyond kMaxSms unrecorded.
#ifdef MOE_TRACE
#define MOE_TRACE_CTA(base, slot)                                                          \
  do {                                                                                     \
    if ((base) && threadIdx.x == 0 && blockIdx.x < kMaxSms)                                \
      (base)[blockIdx.x * kTraceSlots + (slot)] = globaltimer_ns();                        \
  } while (0)
#else
#define MOE_TRACE_CTA(base, slot) (void)0
#endif

// Records `msg` as this thread's last error (moe_b200_last_error) and returns `code`.
int report_error(int code, const char* msg);

// Arguments of the grouped-GEMM kernels (streaming and wide variants, both modes).
struct TileArgs {
  const Plan* plan;
  const int* e_count;
  const int* e_start;
  const int* e_tiles;   // per-expert prefix of this kernel's token tiles (E + 1 entries)
  int E;
  size_t r_pad;
  const float* sa;   // MODE 1: activation scales [56][sa_ld]; MODE 2: C scales [16][r_pad]
  size_t sa_ld;      // leading dimension of sa
  int sa_by_token;   // MODE 1 streaming: sa is hidden_states_scale [56][T], column = the row's token
  const float* sw;   // MODE 1: gemm1_weights_scale [E][32][56]; MODE 2: gemm2_weights_scale [E][56][16]
  uint8_t* c_hi;
  uint8_t* c_lo;
  float* c_scale;
  float* part;       // stream-K partial slots
  int* tile_cnt;     // stream-K per-tile arrival counters (self-resetting)
  const int* row_token;
  const float* row_weight;
  const int* row_nloc;
  const int* tok_nloc;
  const int* tok_rows;
  float* part2;
  OutMap out;
  int* status;
  unsigned long long* trace;   // [kMaxSms][kTraceSlots] of this kernel (written by MOE_TRACE builds)
};




}  // namespace moe
