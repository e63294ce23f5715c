// Work decomposition of the decode kernel.  Plain integer arithmetic shared
// by device code and host-side checks.
//
// Units: u = (seq * num_kv_heads + kv_head) * chunks + chunk, each with T_u
// tiles.  Tiles of all units are flattened unit-major; inside a unit the order
// is split-major with the reference's interleaved assignment (split s owns
// tiles s, s+S, s+2S, ... ; fused_eviction.py:259).
//
// Team w of W gates flattened tiles [range_lo(w, N, W), range_lo(w+1, N, W));
// a unit's tiles [R0, R1] are covered by teams owner(R0) .. owner(R1).  A
// team stores at most two partial states: slot 2w for the first unit of its
// range, 2w+1 for its last unit when that differs and is shared.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define OC_HD __host__ __device__ __forceinline__
#define OC_HD_MEMBER __host__ __device__ __forceinline__
#else
#define OC_HD static inline
#define OC_HD_MEMBER inline
#endif

namespace oc {

// First item of part w when n items are split into W near-equal parts.
OC_HD int64_t range_lo(int64_t w, int64_t n, int64_t W) { return (w * n) / W; }

// The part holding item r (0 <= r < n, W <= n): largest w with range_lo(w) <= r.
OC_HD int64_t range_owner(int64_t r, int64_t n, int64_t W) { return ((r + 1) * W + n - 1) / n - 1; }

// Tile index of the k-th tile (split-major order) of a unit with T tiles and
// S splits: split s holds tiles s, s+S, ...; splits s < T%S hold one more.
OC_HD int split_major_tile(int k, int T, int S) {
  if (S <= 1 || T <= 0) return k;
  const int q = T / S, r = T % S;
  int s, j;
  if (k < r * (q + 1)) {
    s = k / (q + 1);
    j = k % (q + 1);
  } else {
    const int k2 = k - r * (q + 1);
    s = r + k2 / q;
    j = k2 % q;
  }
  return s + j * S;
}

// Iterator over a unit's tiles in split-major order (the sequence
// split_major_tile(0..T-1, T, S) without a division per step).
struct SplitIter {
  int s, j, q, r, S;
  OC_HD_MEMBER void init(int k, int T, int S_) {
    if (S_ <= 1 || T <= 0) {
      S = 1; q = T; r = 0; s = 0; j = k;
      return;
    }
    S = S_; q = T / S_; r = T % S_;
    if (k < r * (q + 1)) {
      s = k / (q + 1);
      j = k % (q + 1);
    } else {
      const int k2 = k - r * (q + 1);
      s = r + k2 / q;
      j = k2 % q;
    }
  }
  OC_HD_MEMBER int tile() const { return s + j * S; }
  OC_HD_MEMBER void next() {
    if (++j >= q + (s < r ? 1 : 0)) {
      ++s;
      j = 0;
    }
  }
};

// Partial-state slot of phase-B warp w for a unit whose first retained rank is R0.
OC_HD int64_t partial_slot(int64_t w, int64_t R0, int64_t Kt, int64_t WB) {
  return (range_lo(w, Kt, WB) >= R0) ? 2 * w : 2 * w + 1;
}

}  // namespace oc
