// Kernel argument structs and launch constants shared by the kernels and the C-ABI launcher.
#pragma once

#include <cstddef>
#include <cstdint>

#include "moe_internal.cuh"

namespace moe {

struct RouteArgs {
  const float* logits;
  const uint16_t* bias;
  const uint8_t* hidden;
  const float* hs_scale;
  uint16_t* out;
  int T, E, offset;
  float rsf;
  int nchunks, num_sms, r_split;
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
  int* e_u1;
  int* e_u2;
  int* row_token;
  float* row_weight;
  uint8_t* a_perm;
  float* sa_perm;
};

struct GemmArgs {
  const Plan* plan;
  const int* e_count;
  const int* e_start;
  const int* e_mt_start;
  const int* e_ustart;
  int E;
  int r_split;
  size_t r_pad;
  const float* sa;   // MODE1: activation scales [56][r_pad]; MODE2: C scales [16][r_pad]
  const float* sw;   // MODE1: gemm1_weights_scale [E][32][56]; MODE2: gemm2_weights_scale [E][56][16]
  // MODE1 outputs
  uint8_t* c_hi;
  uint8_t* c_lo;
  float* c_scale;
  float* part1;
  int* cnt1;
  // MODE2
  const int* row_token;
  const float* row_weight;
  const int* tok_nloc;
  const int* tok_rows;
  float* part2;
  int* cnt2;
  uint16_t* out;
  int* status;
};

constexpr int kStages = 4;
constexpr int kTileBytes = 128 * 128;
constexpr int kStageBytes = 3 * kTileBytes;
constexpr int kGemmThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;

struct GemmSmem {
  uint8_t tiles[kStages][3][kTileBytes];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last_flag;
  int pad;
  float amax[2][128];
};

constexpr size_t kGemmSmemBytes = sizeof(GemmSmem) + 1024;

}  // namespace moe
