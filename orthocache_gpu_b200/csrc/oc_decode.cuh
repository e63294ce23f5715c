// Fused spectral-eviction decode attention for B200 (sm_100a).
//
// One kernel template serves every variant of the reference's hot path
// (j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/):
//   * V1 / V2 zeta-gated split-K decode ........ fused_eviction.py:84-373
//   * V3 Cauchy-Schwarz GQA gate ............... gqa_eviction.py:286-495
//   * paged KV (block-table gather) ............ paged_eviction.py:56-237
//   * mask / zeta scoring only ................. fwht_fused_prototype.py:102-192
//
// Design: a persistent cooperative kernel, one CTA per SM; every warp is an
// independent decoder with its own double-buffered shared-memory ring fed by
// the bulk-copy (TMA) engine, so the per-tile path has no CTA-wide barrier.
//
//   Phase A (K stream).  The tiles of all units (sequence, kv head, query
//   chunk) are flattened (oc_plan.h) and split into equal contiguous ranges,
//   one per warp.  A warp scores each 64-token K tile; for a retained tile it
//   computes the query logits and stores them (fp32, log2 domain) with the
//   tile's flattened index in scratch.  An evicted tile costs one K read.
//   Grid barrier (bounded spin; the launch is cooperative, all CTAs resident).
//   Phase B (V stream).  The Kt retained tiles, in flattened order, are split
//   into equal rank ranges over min(W, Kt) warps, so V traffic is balanced
//   whatever the eviction pattern.  A warp streams V (with the stored logits)
//   of its tiles and keeps an online-softmax state per unit; a unit touched by
//   several warps is merged (log-sum-exp) by the last of them to finish
//   (atomic ticket), so one launch gives the final output.  V of an evicted
//   tile is never read.
//
// Band energies use closed forms of the natural-order 64-point Walsh
// transform along the token axis of the tile (no 64x64 matmul):
//   E_high = sum_{s=32..63} sum_d (W K)[s,d]^2 = 1/2 sum_d sum_{t<32} (K[t,d]-K[t+32,d])^2
//            (row s>=32 of H_64 is [h, -h]);
//   E_low  = sum_{r=1..7}  sum_d (W K)[r,d]^2 = 1/64 sum_d sum_{r=1..7} (H_8 S_d)_r^2
//            with S_d[j] = sum_{t = j mod 8} K[t,d] (row r<8 of H_64 is H_8[r, t mod 8]).
// Lane layout inside a warp: C lanes cover one K row (16 bytes each), RG=32/C
// row groups; lane (rg, c) owns rows rg + RG*m, which hold every pair
// (t, t+32) it needs for E_high; the 8-point transform over the residues
// t mod 8 runs partly in registers and partly across lanes.
//
// Softmax: online, per query head, in the log2 domain (logits pre-scaled by
// log2(e)/sqrt(hd)); m starts at -1e9 and the result is acc / max(l, 1e-9)
// as fused_eviction.py:242-309,369-370.
//
// Every wait is bounded: a wait that runs out sets a status bit and the
// kernel carries on to completion (the outputs of that launch are invalid).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "oc_plan.h"
#include "oc_ptx.cuh"

namespace oc {

enum : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_F8E4M3 = 3 };
// Gate semantics (the reference's three comparison forms):
//   GATE_ZETA_ATTN: evict iff zeta > thr        (attention loops; NaN retains)
//   GATE_ZETA_MASK: retain iff zeta <= thr      (mask helper; NaN evicts)
//   GATE_CS:        evict iff bound <= thr      (V3 Cauchy-Schwarz; NaN retains)
enum : int { GATE_ZETA_ATTN = 0, GATE_ZETA_MASK = 1, GATE_CS = 2 };
enum : int { LAYOUT_LINEAR = 0, LAYOUT_PAGED = 1 };
enum : uint32_t { ST_TIMEOUT = 1u, ST_BAD_PAGE = 2u, ST_BAD_SEQLEN = 4u };

constexpr uint32_t kWaitLimit = 1u << 22;

struct DecodeParams {
  // queries (num_seqs, num_kv_heads*group, head_dim); element strides, dims contiguous
  const void* q;
  int q_dtype;
  int64_t q_seq_stride, q_head_stride;
  // keys / values (byte pointers, byte strides)
  const char* k;
  const char* v;
  int64_t k_seq_stride, k_head_stride, k_tok_stride;
  int64_t v_seq_stride, v_head_stride, v_tok_stride;
  // paged layout: token t of sequence s lives in physical block
  // block_tables[s*bt_seq_stride + (t >> block_shift)], row t & (block_size-1)
  const int32_t* block_tables;
  int64_t bt_seq_stride;
  int64_t k_blk_stride, v_blk_stride;
  int block_shift, num_blocks;
  const int32_t* seq_lens;  // nullable: every sequence has num_tiles*64 tokens
  int layout;
  int num_seqs, num_kv_heads, group, num_tiles, num_splits;
  int gate;
  float thr;
  float scale_log2;  // log2(e)/sqrt(head_dim)
  void* out;
  int out_dtype;
  int64_t out_seq_stride, out_head_stride;
  int8_t* mask;       // (num_seqs, num_kv_heads, num_tiles), nullable
  float* score;       // same shape: zeta or Cauchy-Schwarz bound, nullable
  uint32_t* stats;    // [0] += retained tiles, nullable
  uint32_t* status;   // error bits, non-null
  // workspace (attention only); gbar, cnt_unit and tickets are zero between launches
  uint32_t* gbar;      // [2] grid-barrier arrive / depart counters
  uint32_t* cnt_unit;  // retained tiles per unit (phase A atomics)
  uint32_t* tickets;   // merge tickets per unit
  uint32_t* cnt_warp;  // retained tiles per phase-A warp
  int32_t* list;       // flattened index of each retained tile, at its phase-A position
  float* lg;           // logits of each retained tile at that position: [g][rg][m], GC*64 floats
  float* part;         // partial states [2*W][GC][HD + 4]: acc[HD], m, l
  // shard mode (nullable): write the merged partial state (m, l, unnormalised
  // acc) of each query head instead of the normalised output
  float* sh_m;
  float* sh_l;
  float* sh_acc;
};

// ---------------------------------------------------------------- conversions
// cvt2<N>(src, dst): N consecutive elements at src (shared memory) -> N/2
// float2 pairs (elements 2i, 2i+1).  All conversions are exact.
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int B = 4;
  template <int N> __device__ static void cvt2(const unsigned char* s, float2* f) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 x = *reinterpret_cast<const float4*>(s + 16 * i);
      f[2 * i] = make_float2(x.x, x.y);
      f[2 * i + 1] = make_float2(x.z, x.w);
    }
  }
};
template <> struct Elem<__half> {
  static constexpr int B = 2;
  template <int N> __device__ static void cvt2(const unsigned char* s, float2* f) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) {
      const uint4 x = *reinterpret_cast<const uint4*>(s + 16 * i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) f[4 * i + j] = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    }
  }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int B = 2;
  template <int N> __device__ static void cvt2(const unsigned char* s, float2* f) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) {
      const uint4 x = *reinterpret_cast<const uint4*>(s + 16 * i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        f[4 * i + j] = make_float2(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xffff0000u));
    }
  }
};
template <> struct Elem<__nv_fp8_e4m3> {
  static constexpr int B = 1;
  template <int N> __device__ static void cvt2(const unsigned char* s, float2* f) {
#pragma unroll
    for (int i = 0; i < N / 16; ++i) {
      const uint4 x = *reinterpret_cast<const uint4*>(s + 16 * i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
              static_cast<__nv_fp8x2_storage_t>((w[j] >> (16 * h)) & 0xffffu), __NV_E4M3);
          f[8 * i + 2 * j + h] = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        }
    }
  }
};

__device__ __forceinline__ float load_any(const void* p, int64_t idx, int dt) {
  switch (dt) {
    case DT_F32: return static_cast<const float*>(p)[idx];
    case DT_F16: return __half2float(static_cast<const __half*>(p)[idx]);
    default: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
  }
}

__device__ __forceinline__ void store_any(void* p, int64_t idx, int dt, float x) {
  switch (dt) {
    case DT_F32: static_cast<float*>(p)[idx] = x; break;
    case DT_F16: static_cast<__half*>(p)[idx] = __float2half_rn(x); break;
    default: static_cast<__nv_bfloat16*>(p)[idx] = __float2bfloat16_rn(x); break;
  }
}

// Final write of one query head's merged state.
__device__ __forceinline__ void emit(const DecodeParams& p, int seq, int hq, int d, float m, float l,
                                     float a) {
  if (p.sh_acc != nullptr) {
    const int64_t u = (int64_t)seq * p.num_kv_heads * p.group + hq;
    p.sh_acc[u * (p.out_head_stride) + d] = a;
    if (d == 0) {
      p.sh_m[u] = m;
      p.sh_l[u] = l;
    }
  } else {
    store_any(p.out, (int64_t)seq * p.out_seq_stride + (int64_t)hq * p.out_head_stride + d, p.out_dtype,
              a / fmaxf(l, 1e-9f));
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Reduce-scatter N values over W consecutive lanes (W a power of two <= 32).
// Afterwards lane c (c = lane % W) holds the full sums of value indices
// [c*N/W, (c+1)*N/W) when N >= W, else of index c/(W/N) (replicated).
template <int N, int W>
__device__ __forceinline__ void reduce_scatter(float* v, int c) {
  if constexpr (W > 1) {
    constexpr int off = W / 2;
    if constexpr (N >= 2) {
      constexpr int H = N / 2;
      const bool up = (c & off) != 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = up ? v[i] : v[i + H];
        const float keep = up ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
      reduce_scatter<H, off>(v, c);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
      reduce_scatter<1, off>(v, c);
    }
  }
}

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- config
template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT>
struct Cfg {
  static constexpr int KB = Elem<KT>::B;
  static constexpr int VB = Elem<VT>::B;
  static constexpr int ROWK = HD * KB;
  static constexpr int ROWV = HD * VB;
  static constexpr int C = ROWK / 16;    // lanes per K row (16 bytes each)
  static constexpr int RG = 32 / C;      // row groups per warp
  static constexpr int RPL = 64 / RG;    // rows of a tile per lane
  static constexpr int PAIRS = RPL / 2;  // (t, t+32) pairs per lane
  static constexpr int DPT = 16 / KB;    // head_dim columns per lane
  static constexpr int D2 = DPT / 2;
  static constexpr int RGE = RG < 8 ? RG : 8;
  static constexpr int NRES = 8 / RGE;   // residue classes held per lane
  static constexpr int VCB = DPT * VB;   // bytes of a V row per lane
  static constexpr int ROWMAX = (ATTN && ROWV > ROWK) ? ROWV : ROWK;
  static constexpr int LGB = ATTN ? GC * 64 * 4 : 0;
  static constexpr int SLOT = (64 * ROWMAX + LGB + 127) / 128 * 128;
  static constexpr int RING = 200 * 1024;
  static constexpr int NW0 = RING / (NSLOT * SLOT);
  static constexpr int NW = NW0 > 8 ? 8 : (NW0 < 1 ? 1 : NW0);
  static constexpr int NT = NW * 32;
  static constexpr int MAXU = 2048;  // units per launch (the host batches larger problems)
  static constexpr int MAXW = 1280;  // warps per grid
  static constexpr int OFF_BAR = NW * NSLOT * SLOT;
  static constexpr int OFF_TP = OFF_BAR + 8 * NW * NSLOT;
  static constexpr int OFF_KP = OFF_TP + 4 * (MAXU + 1);
  static constexpr int OFF_PA = OFF_KP + (ATTN ? 4 * (MAXU + 1) : 0);
  static constexpr int OFF_MISC = OFF_PA + (ATTN ? 4 * (MAXW + 1) : 0);
  static constexpr int SMEM = (OFF_MISC + 64 + 127) / 128 * 128;
  static_assert(C >= 1 && C <= 32 && (C & (C - 1)) == 0, "K row bytes must be a power of two in 16..512");
  static_assert(D2 >= 2 && (VCB % 16) == 0, "vector widths");
  static_assert(NW * NSLOT * SLOT >= 4 * NT, "ring doubles as scan scratch");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Block-wide inclusive scan of a[1..n] in place, a[0] = 0; tmp holds blockDim.x ints.
__device__ __noinline__ static void block_scan(int* a, int n, int* tmp) {
  __syncthreads();
  const int nt = blockDim.x, tid = threadIdx.x;
  const int per = (n + nt - 1) / nt;
  const int lo = 1 + tid * per, hi = min(n + 1, lo + per);
  int run = 0;
  for (int i = lo; i < hi; ++i) run += a[i];
  tmp[tid] = run;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int t = 0; t < nt; ++t) {
      const int x = tmp[t];
      tmp[t] = acc;
      acc += x;
    }
  }
  __syncthreads();
  run = tmp[tid];
  for (int i = lo; i < hi; ++i) {
    run += a[i];
    a[i] = run;
  }
  if (tid == 0) a[0] = 0;
  __syncthreads();
}

// Largest i in [0, n] with a[i] <= x (a nondecreasing, a[0] <= x).
__device__ __forceinline__ int upper_index(const int* a, int n, int64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ---------------------------------------------------------------- kernel
template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT>
__global__ void __launch_bounds__(Cfg<KT, VT, HD, GC, ATTN, NSLOT>::NT, 1)
    decode_kernel(const DecodeParams p) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT>;
  constexpr int C = CF::C, RG = CF::RG, RPL = CF::RPL, PAIRS = CF::PAIRS, DPT = CF::DPT, D2 = CF::D2;
  constexpr int RGE = CF::RGE, NRES = CF::NRES, NW = CF::NW, SLOT = CF::SLOT;
  extern __shared__ __align__(128) unsigned char smem[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = lane % C, rg = lane / C;
  const int64_t W = (int64_t)gridDim.x * NW;
  const int64_t wg = (int64_t)blockIdx.x * NW + warp;
  const int nchunks = (p.group + GC - 1) / GC;
  const int U = p.num_seqs * p.num_kv_heads * nchunks;
  const int S = p.num_splits;

  int* tp = reinterpret_cast<int*>(smem + CF::OFF_TP);
  int* kp = reinterpret_cast<int*>(smem + CF::OFF_KP);
  int* pa = reinterpret_cast<int*>(smem + CF::OFF_PA);
  int* misc = reinterpret_cast<int*>(smem + CF::OFF_MISC);
  int* scan_tmp = reinterpret_cast<int*>(smem);  // the ring, while no copy is in flight
  unsigned char* ring = smem + warp * NSLOT * SLOT;
  const uint32_t bars = smem_u32(smem + CF::OFF_BAR) + 8 * warp * NSLOT;

  // ---- tiles per unit, prefix in shared memory
  for (int u = tid; u < U; u += blockDim.x) {
    int T = p.num_tiles;
    if (p.seq_lens != nullptr) {
      const int L = p.seq_lens[u / (p.num_kv_heads * nchunks)];
      if ((L < 0 || (L & 63) || L > p.num_tiles * 64) && blockIdx.x == 0) atomicOr(p.status, ST_BAD_SEQLEN);
      const int lt = L < 0 ? 0 : (L >> 6);
      T = lt < T ? lt : T;
    }
    tp[u + 1] = T;
  }
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NSLOT; ++s) mbar_init(bars + 8 * s, 1);
    mbar_init_fence();
  }
  block_scan(tp, U, scan_tmp);
  const int64_t N = tp[U];

  const uint64_t pol = policy_evict_first();
  uint32_t item = 0;  // tiles this warp has consumed, across both phases

  auto unit_seq = [&](int u) { return u / (p.num_kv_heads * nchunks); };
  auto unit_kvh = [&](int u) { return (u / nchunks) % p.num_kv_heads; };
  auto unit_chunk = [&](int u) { return u % nchunks; };
  auto tile_of = [&](int u, int64_t f) { return (int)split_major_tile(f - tp[u], tp[u + 1] - tp[u], S); };

  // Bulk copy of tile `tile` of unit u (K or V) into ring slot s, plus
  // `extra_bytes` from `extra` (the stored logits) after the tile.
  auto issue = [&](uint32_t s, int u, int tile, bool isv, const float* extra, int extra_bytes) {
    const uint32_t bar = bars + 8 * s;
    const uint32_t dst = smem_u32(ring + s * SLOT);
    const int row = isv ? CF::ROWV : CF::ROWK;
    if (lane == 0) mbar_arrive_expect_tx(bar, 64u * row + extra_bytes);
    __syncwarp();
    const int seq = unit_seq(u), kvh = unit_kvh(u);
    const char* basep = isv ? p.v : p.k;
    const int64_t tok = isv ? p.v_tok_stride : p.k_tok_stride;
    if (p.layout == LAYOUT_LINEAR) {
      const char* base = basep + (int64_t)seq * (isv ? p.v_seq_stride : p.k_seq_stride) +
                         (int64_t)kvh * (isv ? p.v_head_stride : p.k_head_stride);
      if (tok == row) {
        if (lane == 0) bulk_g2s(dst, base + (int64_t)tile * 64 * row, 64u * row, bar, pol);
      } else {
        for (int r = lane; r < 64; r += 32)
          bulk_g2s(dst + r * row, base + ((int64_t)tile * 64 + r) * tok, row, bar, pol);
      }
    } else {
      const int bs = 1 << p.block_shift;
      const int run = bs < 64 ? bs : 64;
      const int nruns = 64 / run;
      const int64_t blk_stride = isv ? p.v_blk_stride : p.k_blk_stride;
      const int64_t head_off = (int64_t)kvh * (isv ? p.v_head_stride : p.k_head_stride);
      for (int i = lane; i < nruns; i += 32) {
        const int t = tile * 64 + i * run;
        int pb = p.block_tables[(int64_t)seq * p.bt_seq_stride + (t >> p.block_shift)];
        if (pb < 0 || pb >= p.num_blocks) {
          atomicOr(p.status, ST_BAD_PAGE);
          pb = 0;
        }
        const char* src = basep + (int64_t)pb * blk_stride + head_off + (int64_t)(t & (bs - 1)) * tok;
        if (tok == row) {
          bulk_g2s(dst + i * run * row, src, (uint32_t)(run * row), bar, pol);
        } else {
          for (int rr = 0; rr < run; ++rr) bulk_g2s(dst + (i * run + rr) * row, src + rr * tok, row, bar, pol);
        }
      }
    }
    if (extra_bytes > 0 && lane == 0) bulk_g2s(dst + 64 * CF::ROWMAX, extra, (uint32_t)extra_bytes, bar, pol);
  };

  auto wait_item = [&](uint32_t it) {
    const uint32_t s = it % NSLOT;
    if (!mbar_wait_bounded(bars + 8 * s, (it / NSLOT) & 1u, kWaitLimit)) {
      if (lane == 0) atomicOr(p.status, ST_TIMEOUT);
      mbar_wait_bounded(bars + 8 * s, (it / NSLOT) & 1u, kWaitLimit);
    }
    return ring + s * SLOT;
  };

  // ======================================================== phase A: K stream
  const int64_t fa = range_lo(wg, N, W), fb = range_lo(wg + 1, N, W);
  const int nA = (int)(fb - fa);
  int kept_local = 0, kept_stat = 0;
  {
    int u_iss = (nA > 0) ? upper_index(tp, U, fa) : 0;
    int u_cur = u_iss;
    int64_t f_iss = fa;
    auto issue_next = [&]() {
      while (f_iss >= tp[u_iss + 1]) ++u_iss;
      issue((uint32_t)(f_iss - fa) % NSLOT, u_iss, tile_of(u_iss, f_iss), false, nullptr, 0);
      ++f_iss;
    };
    for (int i = 0; i < NSLOT && i < nA; ++i) issue_next();

    float2 qv[GC][D2];
    float qmax = 0.f;
    int q_unit = -1;
    int seg_unit = -1, seg_kept = 0;

    for (int i = 0; i < nA; ++i) {
      const int64_t f = fa + i;
      while (f >= tp[u_cur + 1]) ++u_cur;
      const int u = u_cur;
      const int tile = tile_of(u, f);
      if (u != seg_unit) {
        if (ATTN && seg_unit >= 0 && seg_kept && lane == 0) atomicAdd(p.cnt_unit + seg_unit, (uint32_t)seg_kept);
        seg_unit = u;
        seg_kept = 0;
      }
      if constexpr (ATTN) {
        if (u != q_unit) {
          q_unit = u;
          const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
          const int64_t qb = (int64_t)seq * p.q_seq_stride;
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const int hq = chunk * GC + g;
            const bool ok = hq < p.group;
            const int64_t row = qb + (int64_t)(kvh * p.group + hq) * p.q_head_stride + c * DPT;
#pragma unroll
            for (int d = 0; d < D2; ++d)
              qv[g][d] = ok ? make_float2(load_any(p.q, row + 2 * d, p.q_dtype) * p.scale_log2,
                                          load_any(p.q, row + 2 * d + 1, p.q_dtype) * p.scale_log2)
                            : make_float2(0.f, 0.f);
          }
          if (p.gate == GATE_CS) {
            qmax = 0.f;
            for (int g = 0; g < p.group; ++g) {
              const int64_t row = qb + (int64_t)(kvh * p.group + g) * p.q_head_stride + c * DPT;
              float ss = 0.f;
#pragma unroll
              for (int d = 0; d < DPT; ++d) {
                const float x = load_any(p.q, row + d, p.q_dtype);
                ss = fmaf(x, x, ss);
              }
#pragma unroll
              for (int o = C / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
              float qn = sqrtf(ss);
              if (qn < 1e-38f) qn = 0.f;
              if (qn > qmax || qn != qn) qmax = qn;  // NaN propagates like torch.max
            }
          }
        }
      }

      const unsigned char* ts = wait_item(item);

      // ---- band energies
      float2 sres[NRES][D2];
      float2 eh2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < NRES; ++k)
#pragma unroll
        for (int d = 0; d < D2; ++d) sres[k][d] = make_float2(0.f, 0.f);
#pragma unroll
      for (int i2 = 0; i2 < PAIRS; ++i2) {
        float2 a[D2], b[D2];
        Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2) * CF::ROWK + c * 16, a);
        Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2 + 32) * CF::ROWK + c * 16, b);
#pragma unroll
        for (int d = 0; d < D2; ++d) {
          const float2 df = __ffma2_rn(b[d], f2(-1.f), a[d]);
          eh2 = __ffma2_rn(df, df, eh2);
          sres[i2 % NRES][d] = __fadd2_rn(sres[i2 % NRES][d], __fadd2_rn(a[d], b[d]));
        }
      }
      const float eh = warp_sum(eh2.x + eh2.y);
      float score;
      if (p.gate != GATE_CS) {
        // lanes rg and rg+8 (+16, +24) hold the same residue when RG > 8
#pragma unroll
        for (int o = 8 * C; o < 32; o <<= 1)
#pragma unroll
          for (int d = 0; d < D2; ++d) {
            sres[0][d].x += __shfl_xor_sync(0xffffffffu, sres[0][d].x, o);
            sres[0][d].y += __shfl_xor_sync(0xffffffffu, sres[0][d].y, o);
          }
        // 8-point natural-order Walsh transform over residues j = (rg % RGE) + RGE*k:
        // bits of k in registers, bits of rg across lanes
#pragma unroll
        for (int h = 1; h < NRES; h <<= 1)
#pragma unroll
          for (int k = 0; k < NRES; ++k)
            if (!(k & h))
#pragma unroll
              for (int d = 0; d < D2; ++d) {
                const float2 x = sres[k][d], y = sres[k | h][d];
                sres[k][d] = __fadd2_rn(x, y);
                sres[k | h][d] = __ffma2_rn(y, f2(-1.f), x);
              }
#pragma unroll
        for (int bb = 0; (1 << bb) < RGE; ++bb) {
          const int off = C << bb;
          const bool up = (rg >> bb) & 1;
#pragma unroll
          for (int k = 0; k < NRES; ++k)
#pragma unroll
            for (int d = 0; d < D2; ++d) {
              const float yx = __shfl_xor_sync(0xffffffffu, sres[k][d].x, off);
              const float yy = __shfl_xor_sync(0xffffffffu, sres[k][d].y, off);
              sres[k][d].x = up ? (yx - sres[k][d].x) : (sres[k][d].x + yx);
              sres[k][d].y = up ? (yy - sres[k][d].y) : (sres[k][d].y + yy);
            }
        }
        float2 el2 = make_float2(0.f, 0.f);
        if (rg < 8) {
#pragma unroll
          for (int k = 0; k < NRES; ++k) {
            const int j = (rg % RGE) + RGE * k;
            if (j != 0)
#pragma unroll
              for (int d = 0; d < D2; ++d) el2 = __ffma2_rn(sres[k][d], sres[k][d], el2);
          }
        }
        const float el = warp_sum(el2.x + el2.y);
        score = __fdiv_rn(eh * 0.5f, el * (1.f / 64.f) + 1e-6f);
      } else {
        float kn = sqrtf(eh * 0.5f);
        if (kn < 1e-38f) kn = 0.f;
        score = qmax * kn;
      }
      bool keep;
      if (p.gate == GATE_ZETA_ATTN) keep = !(score > p.thr);
      else if (p.gate == GATE_ZETA_MASK) keep = (score <= p.thr);
      else keep = !(score <= p.thr);

      if (lane == 0 && unit_chunk(u) == 0) {
        const int64_t mi = (int64_t)(unit_seq(u) * p.num_kv_heads + unit_kvh(u)) * p.num_tiles + tile;
        if (p.mask) p.mask[mi] = keep ? 1 : 0;
        if (p.score) p.score[mi] = score;
      }
      if (keep) {
        if (unit_chunk(u) == 0) ++kept_stat;
        if constexpr (ATTN) {
          const int64_t pos = fa + kept_local;
          // logits of my rows, reduce-scattered over the C lanes of a row
          constexpr int NV = GC * RPL;
          float lg[NV];
#pragma unroll
          for (int m = 0; m < RPL; ++m) {
            float2 kk[D2];
            Elem<KT>::template cvt2<DPT>(ts + (rg + RG * m) * CF::ROWK + c * 16, kk);
#pragma unroll
            for (int g = 0; g < GC; ++g) {
              float2 acc = make_float2(0.f, 0.f);
#pragma unroll
              for (int d = 0; d < D2; ++d) acc = __ffma2_rn(qv[g][d], kk[d], acc);
              lg[g * RPL + m] = acc.x + acc.y;
            }
          }
          reduce_scatter<NV, C>(lg, c);
          // lane c holds indices [c*2GC, (c+1)*2GC): g = idx / RPL, m = idx % RPL
          float* dstl = p.lg + pos * (GC * 64);
#pragma unroll
          for (int h = 0; h < 2 * GC; h += 2) {
            const int idx = c * 2 * GC + h;
            const int g = idx / RPL, m = idx % RPL;
            *reinterpret_cast<float2*>(dstl + g * 64 + rg * RPL + m) = make_float2(lg[h], lg[h + 1]);
          }
          if (lane == 0) p.list[pos] = (int32_t)f;
          ++kept_local;
          ++seg_kept;
        }
      }
      __syncwarp();
      ++item;
      if (f_iss < fb) issue_next();
    }
    if (ATTN && seg_unit >= 0 && seg_kept && lane == 0) atomicAdd(p.cnt_unit + seg_unit, (uint32_t)seg_kept);
  }
  if (p.stats && lane == 0 && kept_stat) atomicAdd(p.stats, (uint32_t)kept_stat);
  if constexpr (!ATTN) return;

  if constexpr (ATTN) {
    if (lane == 0) p.cnt_warp[wg] = (uint32_t)kept_local;
    // ======================================================== grid barrier
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      atomicAdd(p.gbar, 1u);
      uint32_t n = 0;
      while (ld_acquire_gpu(p.gbar) < gridDim.x) {
        if (++n > kWaitLimit) {
          atomicOr(p.status, ST_TIMEOUT);
          break;
        }
        __nanosleep(64);
      }
    }
    __syncthreads();
    for (int u = tid; u < U; u += blockDim.x) kp[u + 1] = (int)__ldcg(p.cnt_unit + u);
    for (int w = tid; w < W; w += blockDim.x) pa[w + 1] = (int)__ldcg(p.cnt_warp + w);
    block_scan(kp, U, scan_tmp);
    block_scan(pa, (int)W, scan_tmp);
    if (tid == 0) misc[0] = (atomicAdd(p.gbar + 1, 1u) == gridDim.x - 1) ? 1 : 0;
    __syncthreads();
    if (misc[0]) {  // every CTA has read the counters: reset them for the next launch
      for (int u = tid; u < U; u += blockDim.x) p.cnt_unit[u] = 0u;
      if (tid == 0) {
        p.gbar[0] = 0u;
        p.gbar[1] = 0u;
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");

    // ======================================================== phase B: V stream
    const int64_t Kt = pa[W];
    const int64_t WB = Kt < W ? Kt : W;
    // units without a retained tile: zero output (or an empty partial state)
    for (int u = (int)wg; u < U; u += (int)W) {
      if (kp[u + 1] != kp[u]) continue;
      const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
      for (int g = 0; g < GC && chunk * GC + g < p.group; ++g)
        for (int d = lane; d < HD; d += 32) emit(p, seq, kvh * p.group + chunk * GC + g, d, -1e9f, 0.f, 0.f);
    }
    if (wg >= WB) return;
    const int64_t ra = range_lo(wg, Kt, WB), rb = range_lo(wg + 1, Kt, WB);
    const int nB = (int)(rb - ra);

    // retained tile of rank r -> (list position, flattened index)
    auto fetch = [&](int64_t r, int64_t& pos, int64_t& f) {
      const int wa = upper_index(pa, (int)W, r);
      pos = range_lo(wa, N, W) + (r - pa[wa]);
      f = __ldcg(p.list + pos);
    };
    // lanes hold two windows of 32 ranks: [chunk_base, +32) and the next one
    int64_t cpos = 0, cf = 0, npos = 0, nf = 0;
    if (lane < nB) fetch(ra + lane, cpos, cf);
    if (32 + lane < nB) fetch(ra + 32 + lane, npos, nf);
    int chunk_base = 0;
    auto item_at = [&](int j, int64_t& pos, int64_t& f) {  // j in [chunk_base, chunk_base + 64)
      const bool cur = j < chunk_base + 32;
      const int src = (j - chunk_base) & 31;
      pos = __shfl_sync(0xffffffffu, cur ? cpos : npos, src);
      f = __shfl_sync(0xffffffffu, cur ? cf : nf, src);
    };

    int u_iss = 0, u_cur = 0;
    if (nB > 0) {
      int64_t pos0, f0;
      item_at(0, pos0, f0);
      u_iss = u_cur = upper_index(tp, U, f0);
    }
    int j_iss = 0;
    const uint32_t item0 = item;
    auto issue_next_v = [&]() {
      int64_t pos, f;
      item_at(j_iss, pos, f);
      while (f >= tp[u_iss + 1]) ++u_iss;
      issue((item0 + j_iss) % NSLOT, u_iss, tile_of(u_iss, f), true, p.lg + pos * (GC * 64), GC * 64 * 4);
      ++j_iss;
    };
    for (int i = 0; i < NSLOT && i < nB; ++i) issue_next_v();

    float m_run[GC], l_part[GC];
    float2 acc[GC][D2];
    int cur_unit = -1;
    auto reset_state = [&]() {
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        m_run[g] = -1e9f;
        l_part[g] = 0.f;
#pragma unroll
        for (int d = 0; d < D2; ++d) acc[g][d] = make_float2(0.f, 0.f);
      }
    };
    float* part = p.part;
    constexpr int PST = HD + 4;  // floats per (slot, g) partial record

    auto finalize = [&](int u) {
      // sum the row groups' accumulators and the lanes' probability sums
#pragma unroll
      for (int o = C; o < 32; o <<= 1)
#pragma unroll
        for (int g = 0; g < GC; ++g)
#pragma unroll
          for (int d = 0; d < D2; ++d) {
            acc[g][d].x += __shfl_xor_sync(0xffffffffu, acc[g][d].x, o);
            acc[g][d].y += __shfl_xor_sync(0xffffffffu, acc[g][d].y, o);
          }
      float lsum[GC];
#pragma unroll
      for (int g = 0; g < GC; ++g) lsum[g] = warp_sum(l_part[g]);
      const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
      const int gvalid = (p.group - chunk * GC) < GC ? (p.group - chunk * GC) : GC;
      const int64_t R0 = kp[u], R1 = (int64_t)kp[u + 1] - 1;
      const int64_t w0 = range_owner(R0, Kt, WB), w1 = range_owner(R1, Kt, WB);
      if (w0 == w1) {
        if (rg == 0)
          for (int g = 0; g < gvalid; ++g)
#pragma unroll
            for (int d = 0; d < D2; ++d) {
              emit(p, seq, kvh * p.group + chunk * GC + g, c * DPT + 2 * d, m_run[g], lsum[g], acc[g][d].x);
              emit(p, seq, kvh * p.group + chunk * GC + g, c * DPT + 2 * d + 1, m_run[g], lsum[g], acc[g][d].y);
            }
        return;
      }
      const int64_t slot = partial_slot(wg, R0, Kt, WB);
      if (rg == 0)
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          float* rec = part + (slot * GC + g) * PST;
#pragma unroll
          for (int d = 0; d < D2; ++d) *reinterpret_cast<float2*>(rec + c * DPT + 2 * d) = acc[g][d];
          if (c == 0) *reinterpret_cast<float2*>(rec + HD) = make_float2(m_run[g], lsum[g]);
        }
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = (atomicAdd(p.tickets + u, 1u) == (uint32_t)(w1 - w0)) ? 1 : 0;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      __threadfence();
      if (lane == 0) p.tickets[u] = 0u;
      constexpr int NE = (HD + 31) / 32;  // head_dim columns per lane in the merge
      for (int g = 0; g < gvalid; ++g) {
        float M = -INFINITY;
        for (int64_t w = w0 + lane; w <= w1; w += 32) {
          const int64_t sl = (w == w0) ? partial_slot(w0, R0, Kt, WB) : 2 * w;
          M = fmaxf(M, __ldcg(part + (sl * GC + g) * PST + HD));
        }
        M = warp_max(M);
        float lt = 0.f;
        float a[NE];
#pragma unroll
        for (int e = 0; e < NE; ++e) a[e] = 0.f;
#pragma unroll 4
        for (int64_t w = w0; w <= w1; ++w) {
          const int64_t sl = (w == w0) ? partial_slot(w0, R0, Kt, WB) : 2 * w;
          const float* rec = part + (sl * GC + g) * PST;
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec + HD));
          const float wt = exp2f(ml.x - M);
          lt = fmaf(ml.y, wt, lt);
#pragma unroll
          for (int e = 0; e < NE; ++e)
            if (lane + 32 * e < HD) a[e] = fmaf(__ldcg(rec + lane + 32 * e), wt, a[e]);
        }
#pragma unroll
        for (int e = 0; e < NE; ++e)
          if (lane + 32 * e < HD) emit(p, seq, kvh * p.group + chunk * GC + g, lane + 32 * e, M, lt, a[e]);
      }
    };

    reset_state();
    for (int i = 0; i < nB; ++i) {
      int64_t pos, f;
      item_at(i, pos, f);
      while (f >= tp[u_cur + 1]) ++u_cur;
      if (u_cur != cur_unit) {
        if (cur_unit >= 0) finalize(cur_unit);
        reset_state();
        cur_unit = u_cur;
      }
      unsigned char* ts = const_cast<unsigned char*>(wait_item(item));
      float* lgs = reinterpret_cast<float*>(ts + 64 * CF::ROWMAX);
      // per query head: tile max, rescale, probabilities written back in place
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        const float2 mine = reinterpret_cast<const float2*>(lgs + g * 64)[lane];
        const float tmax = warp_max(fmaxf(mine.x, mine.y));
        const float nm = fmaxf(m_run[g], tmax);
        const float alpha = exp2f(m_run[g] - nm);
        m_run[g] = nm;
        const float2 pr = make_float2(exp2f(mine.x - nm), exp2f(mine.y - nm));
        l_part[g] = fmaf(l_part[g], alpha, pr.x + pr.y);
        reinterpret_cast<float2*>(lgs + g * 64)[lane] = pr;
#pragma unroll
        for (int d = 0; d < D2; ++d) acc[g][d] = __fmul2_rn(acc[g][d], f2(alpha));
      }
      __syncwarp();
#pragma unroll
      for (int m4 = 0; m4 < RPL; m4 += 4) {
        float4 pm[GC];
#pragma unroll
        for (int g = 0; g < GC; ++g) pm[g] = *reinterpret_cast<const float4*>(lgs + g * 64 + rg * RPL + m4);
#pragma unroll
        for (int mm = 0; mm < 4; ++mm) {
          float2 vv[D2];
          Elem<VT>::template cvt2<DPT>(ts + (rg + RG * (m4 + mm)) * CF::ROWV + c * CF::VCB, vv);
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const float pv = mm == 0 ? pm[g].x : mm == 1 ? pm[g].y : mm == 2 ? pm[g].z : pm[g].w;
#pragma unroll
            for (int d = 0; d < D2; ++d) acc[g][d] = __ffma2_rn(f2(pv), vv[d], acc[g][d]);
          }
        }
      }
      __syncwarp();
      ++item;
      if (j_iss < nB) issue_next_v();
      // slide the rank window once the process cursor leaves the current 32
      if (i + 1 == chunk_base + 32) {
        cpos = npos;
        cf = nf;
        chunk_base += 32;
        if (chunk_base + 32 + lane < nB) fetch(ra + chunk_base + 32 + lane, npos, nf);
      }
    }
    if (cur_unit >= 0) finalize(cur_unit);
  }
}

template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT>
cudaError_t launch_decode(const DecodeParams& p, int num_sms, cudaStream_t stream) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT>;
  auto kern = decode_kernel<KT, VT, HD, GC, ATTN, NSLOT>;
  int dev = 0;
  cudaGetDevice(&dev);
  static int resident[64] = {0};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (resident[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM);
    if (e != cudaSuccess) return e;
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, CF::NT, CF::SMEM);
    if (e != cudaSuccess) return e;
    if (nb < 1) return cudaErrorInvalidConfiguration;
    resident[dev] = nb;
  }
  const int nchunks = (p.group + GC - 1) / GC;
  const int64_t tiles = (int64_t)p.num_seqs * p.num_kv_heads * nchunks * p.num_tiles;
  // about two tiles per warp, at most one wave of resident CTAs
  const int64_t want = (tiles + 2 * CF::NW - 1) / (2 * CF::NW);
  const int64_t cap = (int64_t)num_sms * resident[dev];
  int64_t grid = want < 1 ? 1 : (want > cap ? cap : want);
  if (grid * CF::NW > CF::MAXW) grid = CF::MAXW / CF::NW;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(CF::NT);
  cfg.dynamicSmemBytes = CF::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = ATTN ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace oc
