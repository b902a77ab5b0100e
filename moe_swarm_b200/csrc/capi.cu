// C ABI of the MoE layer: argument checks, workspace layout, TMA descriptors and the
// launch sequence route -> [scatter] -> GEMM1 -> GEMM2 on the caller's stream.
// No host synchronisation on the forward path; errors are status codes.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"
#include "launch_args.cuh"
#include "moe_internal.cuh"

namespace moe {

cudaError_t route_launch(const RouteArgs& a, cudaStream_t st, int* launches);
cudaError_t wide_prepare();
cudaError_t wide_launch(int mode, int grid, cudaStream_t st, const CUtensorMap& a, const CUtensorMap& a2,
                        const CUtensorMap& b, const TileArgs& g);
cudaError_t stream_prepare();
cudaError_t combine_launch(int T, int grid, cudaStream_t st, const int* tok_nloc, const int* tok_rows,
                           const float* part2, const OutMap& out, unsigned long long* trace);
cudaError_t stream_launch(int mode, int grid, cudaStream_t st, const CUtensorMap& w, const CUtensorMap& t,
                          const CUtensorMap& t2, const TileArgs& g);
cudaError_t stream_fin_launch(int G, cudaStream_t st, const TileArgs& g);
cudaError_t ep_finish_launch(const EpArgs& a, int sms, cudaStream_t st, int* launches);

}  // namespace moe

namespace {

thread_local std::string g_last_error;
thread_local int g_last_launches = 0;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MOE_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Byte matrix [rows, cols] (row stride = cols bytes) read as 128x128-byte tiles, SWIZZLE_128B.
bool encode_u8_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows = 128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool smem_set = false;
};

DeviceInfo& device_info(int dev) {
  static DeviceInfo info[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  DeviceInfo& d = info[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return d;
}

// pre_routed: moe_b200_forward_routed, whose routing_logits / routing_bias are not read.
int check_args(const moe_b200_args* a, bool pre_routed) {
  if (!a) return fail(MOE_B200_ERR_ARG, "null args");
  if (a->num_tokens < 0) return fail(MOE_B200_ERR_ARG, "num_tokens < 0");
  if (a->num_local_experts < 1 || a->num_local_experts > moe::kEG)
    return fail(MOE_B200_ERR_ARG, "num_local_experts must be in [1, 256]");
  if (a->num_tokens == 0) return MOE_B200_OK;
  if ((!pre_routed && (!a->routing_logits || !a->routing_bias)) || !a->hidden_states || !a->hidden_states_scale ||
      !a->gemm1_weights || !a->gemm1_weights_scale || !a->gemm2_weights || !a->gemm2_weights_scale ||
      !a->output)
    return fail(MOE_B200_ERR_ARG, "null tensor pointer");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a->gemm1_weights) || !al16(a->gemm2_weights) || !al16(a->hidden_states) ||
      (!pre_routed && !al16(a->routing_logits)) || !al16(a->output))
    return fail(MOE_B200_ERR_ARG, "weights, hidden states, logits and output must be 16-byte aligned");
  return MOE_B200_OK;
}

moe::RouteArgs make_route_args(const moe_b200_args* a, uint8_t* ws, const moe::Layout& L, int sms) {
  moe::RouteArgs r{};
  r.logits = a->routing_logits;
  r.bias = a->routing_bias;
  r.hidden = a->hidden_states;
  r.hs_scale = a->hidden_states_scale;
  r.out = a->output;
  r.T = a->num_tokens;
  r.E = a->num_local_experts;
  r.offset = a->local_expert_offset;
  r.rsf = a->routed_scaling_factor;
  r.nchunks = L.nchunks;
  r.r_pad = L.r_pad;
  r.plan = reinterpret_cast<moe::Plan*>(ws + L.plan);
  r.route_done = reinterpret_cast<int*>(ws + L.route_done);
  r.topk_idx = reinterpret_cast<int*>(ws + L.topk_idx);
  r.topk_w = reinterpret_cast<float*>(ws + L.topk_w);
  r.tok_nloc = reinterpret_cast<int*>(ws + L.tok_nloc);
  r.tok_le = reinterpret_cast<int*>(ws + L.tok_le);
  r.tok_lw = reinterpret_cast<float*>(ws + L.tok_lw);
  r.tok_rows = reinterpret_cast<int*>(ws + L.tok_rows);
  r.chunk_hist = reinterpret_cast<int*>(ws + L.chunk_hist);
  r.chunk_base = reinterpret_cast<int*>(ws + L.chunk_base);
  r.e_count = reinterpret_cast<int*>(ws + L.e_count);
  r.e_start = reinterpret_cast<int*>(ws + L.e_start);
  r.e_mt_start = reinterpret_cast<int*>(ws + L.e_mt_start);
  r.e_tt = reinterpret_cast<int*>(ws + L.e_tt);
  r.row_token = reinterpret_cast<int*>(ws + L.row_token);
  r.row_weight = reinterpret_cast<float*>(ws + L.row_weight);
  r.row_nloc = reinterpret_cast<int*>(ws + L.row_nloc);
  r.a_perm = ws + L.a_perm;
  r.sa_perm = reinterpret_cast<float*>(ws + L.sa_perm);
  r.trace = reinterpret_cast<unsigned long long*>(ws + L.trace) + 4 * (size_t)moe::kMaxSms * moe::kTraceSlots;
  return r;
}

int prepare(const moe_b200_args* a, void* workspace, size_t ws_bytes, moe::Layout* L, int* dev_out,
            bool pre_routed = false) {
  int rc = check_args(a, pre_routed);
  if (rc) return rc;
  if (!moe::compute_layout(a->num_tokens, a->num_local_experts, L))
    return fail(MOE_B200_ERR_ARG, "bad sizes");
  if (!workspace || ws_bytes < L->total)
    return fail(MOE_B200_ERR_WORKSPACE, "workspace too small: need " + std::to_string(L->total) + " bytes");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(MOE_B200_ERR_ARG, "workspace must be 256-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device_info(dev).major != 10)
    return fail(MOE_B200_ERR_DEVICE, "an sm_100 (B200-class) device is required");
  *dev_out = dev;
  return MOE_B200_OK;
}

// zero_rows: the routing kernels also write the zero output rows of tokens with no local
// expert (moe_b200_route); the full layer leaves them to the combine kernel instead, which
// runs on every SM rather than on the single routing CTA of small batches.
// copy_rows: the permutation also copies the activation rows and their scales into the
// workspace (the token-major GEMMs read them from there); the streaming GEMM1 gathers its token
// rows from hidden_states itself, so the streaming path passes false.
int launch_route(const moe_b200_args* a, uint8_t* ws, const moe::Layout& L, int sms, cudaStream_t st,
                 int* launches, bool zero_rows, const int32_t* pre_idx = nullptr, const float* pre_w = nullptr,
                 bool copy_rows = true) {
  moe::RouteArgs r = make_route_args(a, ws, L, sms);
  if (!zero_rows) r.out = nullptr;
  if (!copy_rows) {
    r.a_perm = nullptr;
    r.sa_perm = nullptr;
  }
  r.pre_idx = pre_idx;
  r.pre_w = pre_w;
  cudaError_t e = moe::route_launch(r, st, launches);
  if (e != cudaSuccess) return cuda_fail(e, "route launch");
  return MOE_B200_OK;
}

}  // namespace

int moe::report_error(int code, const char* msg) { return fail(code, msg); }

extern "C" {

size_t moe_b200_workspace_size(int32_t num_tokens, int32_t num_local_experts) {
  moe::Layout L;
  if (!moe::compute_layout(num_tokens, num_local_experts, &L)) return 0;
  return L.total;
}

int moe_b200_workspace_layout(int32_t num_tokens, int32_t num_local_experts, moe_b200_layout* out) {
  moe::Layout L;
  if (!out || !moe::compute_layout(num_tokens, num_local_experts, &L)) return fail(MOE_B200_ERR_ARG, "bad sizes");
  out->plan = L.plan;
  out->topk_idx = L.topk_idx;
  out->topk_w = L.topk_w;
  out->tok_nloc = L.tok_nloc;
  out->tok_rows = L.tok_rows;
  out->e_count = L.e_count;
  out->e_start = L.e_start;
  out->row_token = L.row_token;
  out->row_weight = L.row_weight;
  out->c_hi = L.c_hi;
  out->c_lo = L.c_lo;
  out->c_scale = L.c_scale;
  out->status = L.status;
  out->trace = L.trace;
  out->r_max = L.r_max;
  out->r_pad = L.r_pad;
  out->total = L.total;
  return MOE_B200_OK;
}

int moe_b200_workspace_init(void* workspace, size_t ws_bytes, int32_t num_tokens, int32_t num_local_experts,
                            void* stream) {
  moe::Layout L;
  if (!moe::compute_layout(num_tokens, num_local_experts, &L)) return fail(MOE_B200_ERR_ARG, "bad sizes");
  if (!workspace || ws_bytes < L.total) return fail(MOE_B200_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(MOE_B200_ERR_ARG, "workspace must be 256-byte aligned");
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(workspace) + L.counters_begin, 0,
                                  L.counters_end - L.counters_begin, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  return MOE_B200_OK;
}

int moe_b200_route(const moe_b200_args* a, void* workspace, size_t ws_bytes, void* stream) {
  moe::Layout L;
  int dev = 0;
  int rc = prepare(a, workspace, ws_bytes, &L, &dev);
  if (rc) return rc;
  if (a->num_tokens == 0) return MOE_B200_OK;
  int launches = 0;
  return launch_route(a, static_cast<uint8_t*>(workspace), L, device_info(dev).sms,
                      static_cast<cudaStream_t>(stream), &launches, true);
}

}  // extern "C"

struct moe_b200_timer {
  std::vector<cudaEvent_t> ev;   // 4 events per call: start, after routing, after GEMM1, after GEMM2
  int used = 0;
  static constexpr int kCap = 4096;
  ~moe_b200_timer() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
};

namespace {

int launch_combine(const moe_b200_args* a, uint8_t* ws, const moe::Layout& L, int sms, cudaStream_t st,
                   int* launches, const moe::OutMap& om) {
  const int T = a->num_tokens;
  const long items = static_cast<long>(moe::kCombineChunks) * T;   // (token, row chunk) pairs
  const int grid = items < 8L * sms ? static_cast<int>(items) : 8 * sms;
  cudaError_t e = moe::combine_launch(T, grid, st, reinterpret_cast<const int*>(ws + L.tok_nloc),
                                      reinterpret_cast<const int*>(ws + L.tok_rows),
                                      reinterpret_cast<const float*>(ws + L.part2), om,
                                      reinterpret_cast<unsigned long long*>(ws + L.trace) +
                                          7 * (size_t)moe::kMaxSms * moe::kTraceSlots);
  if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  ++*launches;
  return MOE_B200_OK;
}

moe::TileArgs tile_args(const moe_b200_args* a, uint8_t* ws, const moe::Layout& L, const moe::OutMap& om) {
  moe::TileArgs s{};
  s.plan = reinterpret_cast<const moe::Plan*>(ws + L.plan);
  s.e_count = reinterpret_cast<const int*>(ws + L.e_count);
  s.e_start = reinterpret_cast<const int*>(ws + L.e_start);
  s.E = a->num_local_experts;
  s.r_pad = L.r_pad;
  s.sa_ld = L.r_pad;
  s.c_hi = ws + L.c_hi;
  s.c_lo = ws + L.c_lo;
  s.c_scale = reinterpret_cast<float*>(ws + L.c_scale);
  s.part = reinterpret_cast<float*>(ws + L.sk_part);
  s.tile_cnt = reinterpret_cast<int*>(ws + L.sk_cnt);
  s.row_token = reinterpret_cast<const int*>(ws + L.row_token);
  s.row_weight = reinterpret_cast<const float*>(ws + L.row_weight);
  s.row_nloc = reinterpret_cast<const int*>(ws + L.row_nloc);
  s.tok_nloc = reinterpret_cast<const int*>(ws + L.tok_nloc);
  s.tok_rows = reinterpret_cast<const int*>(ws + L.tok_rows);
  s.part2 = reinterpret_cast<float*>(ws + L.part2);
  s.out = om;
  s.status = reinterpret_cast<int*>(ws + L.status);
  return s;
}

// om: where the output rows go (null: args->output).
int forward_impl(const moe_b200_args* a, void* workspace, size_t ws_bytes, void* stream,
                 moe_b200_timer* timer, const int32_t* pre_idx = nullptr, const float* pre_w = nullptr,
                 const moe::OutMap* om_in = nullptr) {
  g_last_launches = 0;
  moe::Layout L;
  int dev = 0;
  int rc = prepare(a, workspace, ws_bytes, &L, &dev, pre_idx != nullptr);
  if (rc) return rc;
  moe::OutMap om{};
  if (om_in) {
    om = *om_in;
  } else {
    om.base[0] = a->output;
  }
  om.al32 = 1;
  for (int r = 0; r < moe::kMaxRanks; ++r)
    if (om.base[r] && (reinterpret_cast<uintptr_t>(om.base[r]) & 31u)) om.al32 = 0;
  if (a->num_tokens == 0) return MOE_B200_OK;
  DeviceInfo& di = device_info(dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!di.smem_set) {
    cudaError_t e1 = moe::wide_prepare();
    if (e1 != cudaSuccess) return cuda_fail(e1, "cudaFuncSetAttribute(wide)");
    e1 = moe::stream_prepare();
    if (e1 != cudaSuccess) return cuda_fail(e1, "cudaFuncSetAttribute(stream)");
    di.smem_set = true;
  }
  cudaEvent_t* ev = nullptr;
  if (timer) {
    if (timer->used >= moe_b200_timer::kCap) return fail(MOE_B200_ERR_ARG, "timer full: read it with reset");
    while ((int)timer->ev.size() < 4 * (timer->used + 1)) {
      cudaEvent_t e;
      cudaError_t ce = cudaEventCreate(&e);
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaEventCreate");
      timer->ev.push_back(e);
    }
    ev = timer->ev.data() + 4 * timer->used;
    ++timer->used;
    cudaEventRecord(ev[0], st);
  }
  int launches = 0;
  rc = launch_route(a, ws, L, di.sms, st, &launches, false, pre_idx, pre_w, a->num_tokens > moe::kStreamMaxT);
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[1], st);

  const int E = a->num_local_experts;
  if (a->num_tokens <= moe::kStreamMaxT) {
    CUtensorMap mTok, mW13s, mHi, mLo, mW2s;
    // token rows gathered four at a time from hidden_states (one-row boxes, tile::gather4)
    if (!encode_u8_2d(&mTok, a->hidden_states, moe::kH, static_cast<uint64_t>(a->num_tokens), 1) ||
        !encode_u8_2d(&mW13s, a->gemm1_weights, moe::kH, (uint64_t)E * moe::kN1) ||
        !encode_u8_2d(&mHi, ws + L.c_hi, moe::kI, L.r_pad, moe::kTok) ||
        !encode_u8_2d(&mLo, ws + L.c_lo, moe::kI, L.r_pad, moe::kTok) ||
        !encode_u8_2d(&mW2s, a->gemm2_weights, moe::kI, (uint64_t)E * moe::kH))
      return fail(MOE_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    moe::TileArgs s = tile_args(a, ws, L, om);
    s.e_tiles = reinterpret_cast<const int*>(ws + L.e_tt);
    unsigned long long* trace = reinterpret_cast<unsigned long long*>(ws + L.trace);
    const int grid = di.sms < moe::kMaxSms ? di.sms : moe::kMaxSms;
    moe::TileArgs s1 = s;
    s1.sa = a->hidden_states_scale;   // [56][T], read at each row's token
    s1.sa_ld = static_cast<size_t>(a->num_tokens);
    s1.sa_by_token = 1;
    s1.sw = a->gemm1_weights_scale;
    s1.trace = trace;
    cudaError_t e = moe::stream_launch(1, grid, st, mW13s, mTok, mTok, s1);
    if (e != cudaSuccess) return cuda_fail(e, "stream gemm1 launch");
    ++launches;
    moe::TileArgs s1f = s1;
    s1f.trace = trace + 6 * (size_t)moe::kMaxSms * moe::kTraceSlots;
    e = moe::stream_fin_launch(grid, st, s1f);
    if (e != cudaSuccess) return cuda_fail(e, "stream gemm1 finish launch");
    ++launches;
    if (ev) cudaEventRecord(ev[2], st);
    moe::TileArgs s2 = s;
    s2.sa = reinterpret_cast<const float*>(ws + L.c_scale);
    s2.sw = a->gemm2_weights_scale;
    s2.trace = trace + (size_t)moe::kMaxSms * moe::kTraceSlots;
    e = moe::stream_launch(2, grid, st, mW2s, mHi, mLo, s2);
    if (e != cudaSuccess) return cuda_fail(e, "stream gemm2 launch");
    ++launches;
    rc = launch_combine(a, ws, L, di.sms, st, &launches, om);
    if (rc) return rc;
    if (ev) cudaEventRecord(ev[3], st);
    g_last_launches = launches;
    return MOE_B200_OK;
  }
  // wide (token-major) kernels for large T
  CUtensorMap mA1, mW13, mChi, mClo, mW2;
  if (!encode_u8_2d(&mA1, ws + L.a_perm, moe::kH, L.r_pad, 128) ||
      !encode_u8_2d(&mW13, a->gemm1_weights, moe::kH, (uint64_t)E * moe::kN1) ||
      !encode_u8_2d(&mChi, ws + L.c_hi, moe::kI, L.r_pad, 128) ||
      !encode_u8_2d(&mClo, ws + L.c_lo, moe::kI, L.r_pad, 128) ||
      !encode_u8_2d(&mW2, a->gemm2_weights, moe::kI, (uint64_t)E * moe::kH))
    return fail(MOE_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  moe::TileArgs w = tile_args(a, ws, L, om);
  unsigned long long* trace = reinterpret_cast<unsigned long long*>(ws + L.trace);
  const int grid = di.sms < moe::kMaxSms ? di.sms : moe::kMaxSms;
  moe::TileArgs w1 = w;
  w1.e_tiles = reinterpret_cast<const int*>(ws + L.e_mt_start);
  w1.sa = reinterpret_cast<const float*>(ws + L.sa_perm);
  w1.sw = a->gemm1_weights_scale;
  w1.trace = trace + 2 * (size_t)moe::kMaxSms * moe::kTraceSlots;
  cudaError_t e = moe::wide_launch(1, grid, st, mA1, mA1, mW13, w1);
  if (e != cudaSuccess) return cuda_fail(e, "wide gemm1 launch");
  ++launches;
  if (ev) cudaEventRecord(ev[2], st);
  moe::TileArgs w2 = w;
  w2.e_tiles = reinterpret_cast<const int*>(ws + L.e_mt_start);
  w2.sa = reinterpret_cast<const float*>(ws + L.c_scale);
  w2.sw = a->gemm2_weights_scale;
  w2.trace = trace + 3 * (size_t)moe::kMaxSms * moe::kTraceSlots;
  e = moe::wide_launch(2, grid, st, mChi, mClo, mW2, w2);
  if (e != cudaSuccess) return cuda_fail(e, "wide gemm2 launch");
  ++launches;
  rc = launch_combine(a, ws, L, di.sms, st, &launches, om);
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[3], st);
  g_last_launches = launches;
  return MOE_B200_OK;
}

}  // namespace

extern "C" {

int moe_b200_forward(const moe_b200_args* a, void* workspace, size_t ws_bytes, void* stream) {
  return forward_impl(a, workspace, ws_bytes, stream, nullptr);
}

int moe_b200_forward_routed(const moe_b200_args* a, const int32_t* topk_idx, const float* topk_w,
                            void* workspace, size_t ws_bytes, void* stream) {
  if (a && a->num_tokens > 0 && (!topk_idx || !topk_w)) return fail(MOE_B200_ERR_ARG, "null topk_idx / topk_w");
  return forward_impl(a, workspace, ws_bytes, stream, nullptr, topk_idx, topk_w);
}

int moe_b200_forward_ep(const moe_b200_args* a, const moe_b200_ep* ep, void* workspace, size_t ws_bytes,
                        void* stream) {
  if (!a || !ep) return fail(MOE_B200_ERR_ARG, "null args or ep");
  const int N = ep->world, T = a->num_tokens;
  if (N < 1 || N > MOE_B200_MAX_RANKS || ep->rank < 0 || ep->rank >= N)
    return fail(MOE_B200_ERR_ARG, "ep: world must be in [1, 8] and rank in [0, world)");
  if (T < 0 || ep->shard_tokens < 0 || static_cast<int64_t>(ep->shard_tokens) * N != T)
    return fail(MOE_B200_ERR_ARG, "ep: shard_tokens * world must equal num_tokens");
  if (ep->epoch == 0) return fail(MOE_B200_ERR_ARG, "ep: epoch counts calls from 1");
  if (T == 0) return MOE_B200_OK;
  if (!ep->out_shard || (reinterpret_cast<uintptr_t>(ep->out_shard) & 15u))
    return fail(MOE_B200_ERR_ARG, "ep: out_shard must be a 16-byte aligned pointer");
  for (int r = 0; r < N; ++r)
    if (!ep->recv[r] || !ep->signal[r] || (reinterpret_cast<uintptr_t>(ep->recv[r]) & 15u))
      return fail(MOE_B200_ERR_ARG, "ep: recv[r] (16-byte aligned) and signal[r] are required for every rank");
  moe_b200_args a2 = *a;
  a2.output = static_cast<uint16_t*>(ep->out_shard);   // passes the argument check; rows go through the map
  const int phase = static_cast<int>(ep->epoch & 1u);
  const size_t slot = static_cast<size_t>(ep->shard_tokens) * moe::kH;   // bf16 elements
  moe::OutMap om{};
  for (int r = 0; r < N; ++r)
    om.base[r] = static_cast<uint16_t*>(ep->recv[r]) + static_cast<size_t>(phase) * N * slot;
  om.shard = ep->shard_tokens;
  om.slot_rows = ep->rank * ep->shard_tokens;
  int rc = forward_impl(&a2, workspace, ws_bytes, stream, nullptr, nullptr, nullptr, &om);
  if (rc) return rc;
  moe::Layout L;
  moe::compute_layout(T, a->num_local_experts, &L);
  int dev = 0;
  cudaGetDevice(&dev);
  moe::EpArgs e{};
  for (int r = 0; r < N; ++r) e.signal[r] = ep->signal[r];
  e.recv = static_cast<const uint16_t*>(ep->recv[ep->rank]) + static_cast<size_t>(phase) * N * slot;
  e.out = static_cast<uint16_t*>(ep->out_shard);
  e.world = N;
  e.rank = ep->rank;
  e.shard = ep->shard_tokens;
  e.phase = phase;
  e.epoch = ep->epoch;
  e.wait_ns = ep->wait_limit_us ? static_cast<unsigned long long>(ep->wait_limit_us) * 1000ull : moe::kWaitLimitNs;
  e.status = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + L.status);
  int launches = 0;
  cudaError_t ce = moe::ep_finish_launch(e, device_info(dev).sms, static_cast<cudaStream_t>(stream), &launches);
  g_last_launches += launches;
  if (ce != cudaSuccess) return cuda_fail(ce, "ep signal / reduce launch");
  return MOE_B200_OK;
}

moe_b200_timer* moe_b200_timer_create(void) { return new moe_b200_timer(); }

void moe_b200_timer_destroy(moe_b200_timer* t) { delete t; }

int moe_b200_forward_timed(const moe_b200_args* a, void* workspace, size_t ws_bytes, void* stream,
                           moe_b200_timer* timer) {
  if (!timer) return fail(MOE_B200_ERR_ARG, "null timer");
  return forward_impl(a, workspace, ws_bytes, stream, timer);
}

int moe_b200_timer_read(moe_b200_timer* t, float* stage_ms, int32_t* calls, int32_t reset) {
  if (!t || !stage_ms || !calls) return fail(MOE_B200_ERR_ARG, "null argument");
  stage_ms[0] = stage_ms[1] = stage_ms[2] = 0.f;
  *calls = t->used;
  if (t->used > 0) {
    cudaError_t e = cudaEventSynchronize(t->ev[4 * (t->used - 1) + 3]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    for (int i = 0; i < t->used; ++i)
      for (int s = 0; s < 3; ++s) {
        float ms = 0.f;
        e = cudaEventElapsedTime(&ms, t->ev[4 * i + s], t->ev[4 * i + s + 1]);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
        stage_ms[s] += ms;
      }
  }
  if (reset) t->used = 0;
  return MOE_B200_OK;
}

int moe_b200_device_status(void* workspace, size_t ws_bytes, int32_t num_tokens, int32_t num_local_experts,
                           void* stream, int32_t clear) {
  moe::Layout L;
  if (!moe::compute_layout(num_tokens, num_local_experts, &L)) return -fail(MOE_B200_ERR_ARG, "bad sizes");
  if (!workspace || ws_bytes < L.total) return -fail(MOE_B200_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return -fail(MOE_B200_ERR_ARG, "workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  int* p = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + L.status);
  cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(p, 0, sizeof(int), st);
  if (e != cudaSuccess) return -cuda_fail(e, "device status");
  return v;
}

const char* moe_b200_last_error(void) { return g_last_error.c_str(); }

int moe_b200_last_launch_count(void) { return g_last_launches; }

}  // extern "C"
