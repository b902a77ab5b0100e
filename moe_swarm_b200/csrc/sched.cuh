// Work distribution of the persistent grouped-GEMM kernels: data-parallel whole tiles, then
// a stream-K tail.
//
// Tiles [0, dp) are handed out round-robin (tile t to CTA t mod G), whole: consecutive tiles
// -- the token tiles of one weight tile -- run at the same time on neighbouring CTAs and
// share the weight tile through L2.  The remaining 1-2 waves of tiles, [dp, tiles), are
// split stream-K: their W = (tiles - dp) * KB K-blocks are cut into G equal contiguous
// ranges, CTA c owning [w0(c), w0(c+1)) with w0(c) = floor(c*W/G), so every CTA streams the
// same number of K-blocks (+-1) whatever the tile count.  In the decode regime, where the
// routed experts give fewer tiles than SMs, everything is stream-K and all 148 SMs stream
// weights.  A tile split across CTAs is finished by its last contributor to arrive (wide
// kernels), by its first contributor, which in this order reaches it last (streaming GEMM2), or
// by stream_fin1_kernel after the GEMM (streaming GEMM1); each sums the partial accumulators of
// the contributing CTAs in CTA order (deterministic).  Only a CTA's
// first and last stream-K tile can be partial, so each CTA owns two partial slots: 2c (its
// first) and 2c+1 (its last).
#pragma once

#include <cstdint>

namespace moe {

struct Sched {
  int tiles;     // total tiles
  int dp;        // tiles [0, dp) are data-parallel
  int G;         // CTAs
  int KB;        // K-blocks per tile
  long long W;   // stream-K K-blocks: (tiles - dp) * KB

  __device__ __forceinline__ void init(int tiles_, int G_, int KB_) {
    tiles = tiles_;
    G = G_;
    KB = KB_;
    dp = tiles >= 2 * G ? (tiles / G - 1) * G : 0;
    W = static_cast<long long>(tiles - dp) * KB;
  }
  __device__ __forceinline__ long long w0(int c) const { return static_cast<long long>(c) * W / G; }
  __device__ __forceinline__ bool has_work(int c) const { return c < dp || w0(c) != w0(c + 1); }
  // CTA whose stream-K range holds work index x
  __device__ __forceinline__ int owner(long long x) const { return static_cast<int>(((x + 1) * G - 1) / W); }
  // contributors to stream-K tile `tile` (absolute index, tile >= dp)
  __device__ __forceinline__ int first_cta(int tile) const {
    return owner(static_cast<long long>(tile - dp) * KB);
  }
  __device__ __forceinline__ int last_cta(int tile) const {
    return owner(static_cast<long long>(tile - dp) * KB + KB - 1);
  }
  // partial slot of CTA c for stream-K tile `tile` (c must contribute to it)
  __device__ __forceinline__ int slot(int c, int tile) const {
    return 2 * c + ((w0(c) / KB) == (tile - dp) ? 0 : 1);
  }
};

// Iterates the segments (tile, k0, k1) of CTA c in order: its data-parallel tiles, then its
// stream-K range.  `partial` is set for a stream-K segment that is not a whole tile.
struct SegIter {
  const Sched& s;
  int c;
  int dp_next;
  long long w, wend;
  __device__ __forceinline__ SegIter(const Sched& s_, int c_)
      : s(s_), c(c_), dp_next(c_), w(s_.w0(c_)), wend(s_.w0(c_ + 1)) {}
  __device__ __forceinline__ bool next(int& tile, int& k0, int& k1) {
    if (dp_next < s.dp) {
      tile = dp_next;
      k0 = 0;
      k1 = s.KB;
      dp_next += s.G;
      return true;
    }
    if (w >= wend) return false;
    tile = s.dp + static_cast<int>(w / s.KB);
    k0 = static_cast<int>(w % s.KB);
    const long long rem = wend - w;
    k1 = (s.KB - k0) < rem ? s.KB : static_cast<int>(k0 + rem);
    w += k1 - k0;
    return true;
  }
};

}  // namespace moe
