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
#include <type_traits>

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

// Unroll factors of the per-tile row loops (instruction-cache footprint).
#ifndef OC_UNROLL_PAIRS
#define OC_UNROLL_PAIRS 2
#endif
#ifndef OC_UNROLL_PV
#define OC_UNROLL_PV 2
#endif
constexpr int kUnrollPairs = OC_UNROLL_PAIRS;
#ifndef OC_MAX_WARPS_PER_CTA
#define OC_MAX_WARPS_PER_CTA 8
#endif
constexpr int kMaxWarpsPerCta = OC_MAX_WARPS_PER_CTA;
#ifndef OC_COPY_SPLIT
#define OC_COPY_SPLIT 1
#endif
constexpr int kCopySplit = OC_COPY_SPLIT;
#ifdef OC_PROBE_NO_GATE_MATH
constexpr bool kGateMath = false;  // measurement probe: stream tiles, skip the band energies
#else
constexpr bool kGateMath = true;
#endif
constexpr int kUnrollPV = OC_UNROLL_PV;

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
  static constexpr int NWC = NW0 > kMaxWarpsPerCta ? kMaxWarpsPerCta : NW0;
  static constexpr int NW = NWC < 1 ? 1 : NWC;
  static constexpr int NT = NW * 32;
  static constexpr int MAXU = 2048;  // units per launch (the host batches larger problems)
  static constexpr int MAXW = 1280;  // warps per grid
  static constexpr int OFF_BAR = NW * NSLOT * SLOT;
  static constexpr int OFF_TP = OFF_BAR;
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
// TC: 16-bit K/V (and queries of the K dtype), head_dim >= 64: band energies,
// logits and PV on the tensor cores (mma.sync m16n8k16), tiles stored
// swizzled in shared memory.  Otherwise the same math runs on CUDA cores.
template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT, bool TC>
__global__ void __launch_bounds__(Cfg<KT, VT, HD, GC, ATTN, NSLOT>::NT, 1)
    decode_kernel(const DecodeParams p) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT>;
  constexpr int C = CF::C, RG = CF::RG, RPL = CF::RPL, PAIRS = CF::PAIRS, DPT = CF::DPT, D2 = CF::D2;
  constexpr int RGE = CF::RGE, NRES = CF::NRES, NW = CF::NW, SLOT = CF::SLOT;
  extern __shared__ __align__(128) unsigned char smem[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = lane % C, rg = lane / C;
  static_assert(!TC || (CF::KB == 2 && CF::VB == 2 && HD >= 64 && GC <= 8), "tensor-core path");
  constexpr bool KBF16 = TC && (sizeof(KT) == 2) && !std::is_same<KT, __half>::value;
  const int g8 = lane >> 2, t4 = lane & 3;  // mma fragment coordinates
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
  block_scan(tp, U, scan_tmp);
  const int64_t N = tp[U];

  const uint64_t pol = policy_evict_first();
  uint32_t item = 0;  // tiles this warp has consumed, across both phases

  auto unit_seq = [&](int u) { return u / (p.num_kv_heads * nchunks); };
  auto unit_kvh = [&](int u) { return (u / nchunks) % p.num_kv_heads; };
  auto unit_chunk = [&](int u) { return u % nchunks; };
  auto tile_of = [&](int u, int64_t f) { return split_major_tile((int)(f - tp[u]), tp[u + 1] - tp[u], S); };

  // Bulk copy of tile `tile` of unit u (K or V) into ring slot s, plus
  // `extra_bytes` from `extra` (the stored logits) after the tile.
  // Byte offset of tile byte o (row-major, `row` bytes per row) in shared
  // memory: on the tensor-core path the 16-byte chunks of each row are XORed
  // with (row & 7), so ldmatrix reads of 8 rows hit 8 distinct bank groups.
  auto swz = [&](int o, int r) -> int {
    if constexpr (TC) {
      return o ^ ((r & 7) << 4);
    } else {
      return o;
    }
  };
  // row of tile byte o (row sizes are compile-time powers of two)
  auto row_of = [&](int o, bool isv) -> int { return isv ? o / CF::ROWV : o / CF::ROWK; };
  // smem address of (token, dim) of a 16-bit tile with `row` bytes per row
  auto tc_addr = [&](uint32_t base, int tok, int dim, int row) -> uint32_t {
    return base + tok * row + ((((dim * 2) >> 4) ^ (tok & 7)) << 4);
  };

  // Asynchronous copy (16-byte cp.async per lane, one commit group per item)
  // of tile `tile` of unit u (K or V) into ring slot s, plus `extra_bytes`
  // from `extra` (the stored logits) after the tile.  The warp's groups
  // complete in order, so waiting for "at most NSLOT-1 pending" makes the
  // oldest item resident.
  auto issue = [&](uint32_t s, int u, int tile, bool isv, const float* extra, int extra_bytes) {
#ifdef OC_PROBE_NO_LOAD
    cp_async_commit();  // measurement probe: no memory traffic, the slot keeps stale data
    return;
#endif
    const uint32_t dst = smem_u32(ring + s * SLOT);
    const int row = isv ? CF::ROWV : CF::ROWK;
    const int tbytes = 64 * row;
    const int seq = unit_seq(u), kvh = unit_kvh(u);
    const char* basep = isv ? p.v : p.k;
    const int64_t tok = isv ? p.v_tok_stride : p.k_tok_stride;
    if (p.layout == LAYOUT_LINEAR) {
      const char* base = basep + (int64_t)seq * (isv ? p.v_seq_stride : p.k_seq_stride) +
                         (int64_t)kvh * (isv ? p.v_head_stride : p.k_head_stride) + (int64_t)tile * 64 * tok;
      if (tok == row) {
#pragma unroll 8
        for (int o = lane * 16; o < tbytes; o += 512) cp_async16(dst + swz(o, row_of(o, isv)), base + o, pol);
      } else {
#pragma unroll 8
        for (int o = lane * 16; o < tbytes; o += 512) {
          const int r = row_of(o, isv), col = o - r * row;
          cp_async16(dst + swz(o, r), base + (int64_t)r * tok + col, pol);
        }
      }
    } else {
      const int shift = p.block_shift;
      const int64_t blk_stride = isv ? p.v_blk_stride : p.k_blk_stride;
      const char* base = basep + (int64_t)kvh * (isv ? p.v_head_stride : p.k_head_stride);
      const int32_t* bt = p.block_tables + (int64_t)seq * p.bt_seq_stride;
      const int t0 = tile * 64;
      const int first = t0 >> shift;
      const int npages = ((t0 + 63) >> shift) - first + 1;
      int mine = 0;  // physical block of page (first + lane)
      if (lane < npages && npages <= 32) {
        mine = bt[first + lane];
        if (mine < 0 || mine >= p.num_blocks) {
          atomicOr(p.status, ST_BAD_PAGE);
          mine = 0;
        }
      }
      const int bmask = (1 << shift) - 1;
#pragma unroll 4
      for (int o = lane * 16; o < tbytes; o += 512) {
        const int r = row_of(o, isv), col = o - r * row;
        const int t = t0 + r;
        int pb;
        if (npages <= 32) {
          pb = __shfl_sync(0xffffffffu, mine, (t >> shift) - first);
        } else {
          pb = bt[t >> shift];
          if (pb < 0 || pb >= p.num_blocks) {
            atomicOr(p.status, ST_BAD_PAGE);
            pb = 0;
          }
        }
        cp_async16(dst + swz(o, r), base + (int64_t)pb * blk_stride + (int64_t)(t & bmask) * tok + col, pol);
      }
    }
    for (int o = lane * 16; o < extra_bytes; o += 512)
      cp_async16(dst + 64 * CF::ROWMAX + o, reinterpret_cast<const char*>(extra) + o, pol);
    cp_async_commit();
  };

  auto wait_item = [&](uint32_t it) {
    cp_async_wait<NSLOT - 1>();
    __syncwarp();
    return ring + (it % NSLOT) * SLOT;
  };

  float qmax = 0.f;  // max_g |q_g| of the current unit (Cauchy-Schwarz gate)
  // ---- tensor-core constants: A fragments of W rows 1..7 (E_low) and of +-I (K[t] - K[t+32])
  uint32_t aW[TC ? 4 : 1][4], aPos[4], aNeg[4];
  if constexpr (TC) {
    const uint32_t P8 = KBF16 ? 0x3E00u : 0x3000u, N8 = KBF16 ? 0xBE00u : 0xB000u;
    const uint32_t ONE = KBF16 ? 0x3F80u : 0x3C00u, MONE = KBF16 ? 0xBF80u : 0xBC00u;
    auto w = [&](int r, int tk) -> uint32_t {
      if (r < 1 || r > 7) return 0u;  // row 0 (DC) and rows >= 8 do not enter E_low
      return (__popc(r & tk) & 1) ? N8 : P8;
    };
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int c0 = 16 * ks + 2 * t4;
      aW[ks][0] = w(g8, c0) | (w(g8, c0 + 1) << 16);
      aW[ks][1] = 0u;
      aW[ks][2] = w(g8, c0 + 8) | (w(g8, c0 + 9) << 16);
      aW[ks][3] = 0u;
    }
    const uint32_t ip = (g8 == 2 * t4 ? ONE : 0u) | ((g8 == 2 * t4 + 1 ? ONE : 0u) << 16);
    const uint32_t in = (g8 == 2 * t4 ? MONE : 0u) | ((g8 == 2 * t4 + 1 ? MONE : 0u) << 16);
    aPos[0] = ip; aPos[1] = 0u; aPos[2] = 0u; aPos[3] = ip;
    aNeg[0] = in; aNeg[1] = 0u; aNeg[2] = 0u; aNeg[3] = in;
  }
  // E_low = sum (W K)[1..7]^2 and E_high = 1/2 sum (K[t]-K[t+32])^2 with mma:
  // B = the K tile (tokens x head_dim), 16 columns per step.
  auto tc_gate = [&](const unsigned char* ts) -> float {
    const uint32_t base = smem_u32(ts);
    float2 el2 = make_float2(0.f, 0.f), eh2 = make_float2(0.f, 0.f);
#pragma unroll 2
    for (int np = 0; np < HD / 16; ++np) {
      float cl[2][4] = {}, cd[2][2][4] = {};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t b[4];
        ldsm_x4_t(tc_addr(base, 16 * ks + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * np + ((lane >> 4) & 1) * 8,
                          CF::ROWK), b);
        mma16816<KBF16>(cl[0], aW[ks], b[0], b[1]);
        mma16816<KBF16>(cl[1], aW[ks], b[2], b[3]);
        mma16816<KBF16>(cd[ks & 1][0], ks < 2 ? aPos : aNeg, b[0], b[1]);
        mma16816<KBF16>(cd[ks & 1][1], ks < 2 ? aPos : aNeg, b[2], b[3]);
      }
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const float2 x = make_float2(cl[n][0], cl[n][1]);
        el2 = __ffma2_rn(x, x, el2);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const float2 y0 = make_float2(cd[mt][n][0], cd[mt][n][1]);
          const float2 y1 = make_float2(cd[mt][n][2], cd[mt][n][3]);
          eh2 = __ffma2_rn(y0, y0, eh2);
          eh2 = __ffma2_rn(y1, y1, eh2);
        }
      }
    }
    const float eh = warp_sum(eh2.x + eh2.y);
    if (p.gate != GATE_CS) {
      const float el = warp_sum(el2.x + el2.y);
      return __fdiv_rn(eh * 0.5f, el + 1e-6f);
    }
    float kn = sqrtf(eh * 0.5f);
    if (kn < 1e-38f) kn = 0.f;
    return qmax * kn;
  };

  // ======================================================== phase A: K stream
#ifdef OC_PROBE_SPAN
  uint64_t span_t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(span_t0));
#endif
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
    for (int i = 0; i < NSLOT; ++i) {
      if (i < nA) issue_next(); else cp_async_commit();
    }

    float2 qv[TC ? 1 : GC][D2];
    uint32_t qf[TC ? HD / 16 : 1][2];  // q as mma B fragments (dims x queries), raw 16-bit
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
          if constexpr (TC) {
            const int hq = chunk * GC + g8;
            const bool ok = g8 < GC && hq < p.group;
            const uint16_t* qrow = static_cast<const uint16_t*>(p.q) + qb + (int64_t)(kvh * p.group + hq) * p.q_head_stride;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
              qf[ks][0] = ok ? (uint32_t)qrow[16 * ks + 2 * t4] | ((uint32_t)qrow[16 * ks + 2 * t4 + 1] << 16) : 0u;
              qf[ks][1] = ok ? (uint32_t)qrow[16 * ks + 2 * t4 + 8] | ((uint32_t)qrow[16 * ks + 2 * t4 + 9] << 16) : 0u;
            }
          } else {
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
          }
          if (p.gate == GATE_CS) {
            qmax = 0.f;
            for (int g = 0; g < p.group; ++g) {
              const int64_t row = qb + (int64_t)(kvh * p.group + g) * p.q_head_stride;
              float ss = 0.f;
              for (int d = lane; d < HD; d += 32) {
                const float x = load_any(p.q, row + d, p.q_dtype);
                ss = fmaf(x, x, ss);
              }
              ss = warp_sum(ss);
              float qn = sqrtf(ss);
              if (qn < 1e-38f) qn = 0.f;
              if (qn > qmax || qn != qn) qmax = qn;  // NaN propagates like torch.max
            }
          }
        }
      }

#ifdef OC_PROBE_TIMING
      const uint32_t t_w0 = (uint32_t)clock();
#endif
      const unsigned char* ts = wait_item(item);
#ifdef OC_PROBE_TIMING
      const uint32_t t_w1 = (uint32_t)clock();
#endif

      // ---- band energies
      float score;
      if constexpr (TC) {
        score = tc_gate(ts);
      } else {
        float2 sres[NRES][D2];
        float2 ehd[D2];  // one E_high accumulator per column pair: independent FMA chains
#pragma unroll
        for (int d = 0; d < D2; ++d) ehd[d] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < NRES; ++k)
#pragma unroll
          for (int d = 0; d < D2; ++d) sres[k][d] = make_float2(0.f, 0.f);
#pragma unroll kUnrollPairs
        for (int i0 = 0; i0 < (kGateMath ? PAIRS : 0); i0 += NRES) {
#pragma unroll
          for (int k = 0; k < NRES; ++k) {
            const int i2 = i0 + k;
            float2 a[D2], b[D2];
            Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2) * CF::ROWK + c * 16, a);
            Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2 + 32) * CF::ROWK + c * 16, b);
#pragma unroll
            for (int d = 0; d < D2; ++d) {
              const float2 df = __ffma2_rn(b[d], f2(-1.f), a[d]);
              ehd[d] = __ffma2_rn(df, df, ehd[d]);
              sres[k][d] = __fadd2_rn(sres[k][d], __fadd2_rn(a[d], b[d]));
            }
          }
        }
        float2 eh2 = ehd[0];
#pragma unroll
        for (int d = 1; d < D2; ++d) eh2 = __fadd2_rn(eh2, ehd[d]);
        const float eh = warp_sum(eh2.x + eh2.y);
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
      }
      bool keep;
      if (p.gate == GATE_ZETA_ATTN) keep = !(score > p.thr);
      else if (p.gate == GATE_ZETA_MASK) keep = (score <= p.thr);
      else keep = !(score <= p.thr);

#if !defined(OC_PROBE_TIMING) && !defined(OC_PROBE_SPAN)
      if (lane == 0 && unit_chunk(u) == 0) {
        const int64_t mi = (int64_t)(unit_seq(u) * p.num_kv_heads + unit_kvh(u)) * p.num_tiles + tile;
        if (p.mask) p.mask[mi] = keep ? 1 : 0;
        if (p.score) p.score[mi] = score;
      }
#endif
      if (keep) {
        if (unit_chunk(u) == 0) ++kept_stat;
        if constexpr (ATTN) {
          const int64_t pos = fa + kept_local;
          if constexpr (TC) {
            // logits = K (tokens x dims) * q (dims x queries): 4 token tiles of 16
            const uint32_t base = smem_u32(ts);
            float cq[4][4] = {};
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
              for (int mt = 0; mt < 4; ++mt) {
                uint32_t a4[4];
                ldsm_x4(tc_addr(base, 16 * mt + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * ks + ((lane >> 4) & 1) * 8,
                                CF::ROWK), a4);
                mma16816<KBF16>(cq[mt], a4, qf[ks][0], qf[ks][1]);
              }
            // C(token, query): lane holds tokens 16mt+g8 (+8), queries 2t4, 2t4+1
            float* dstl = p.lg + pos * (GC * 64);
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int qq = 2 * t4 + (j & 1), tk = 16 * mt + g8 + (j >> 1) * 8;
                if (qq < GC) dstl[qq * 64 + tk] = cq[mt][j] * p.scale_log2;
              }
          } else {
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
          }
          if (lane == 0) p.list[pos] = (int32_t)f;
          ++kept_local;
          ++seg_kept;
        }
      }
      __syncwarp();
      ++item;
#ifdef OC_PROBE_TIMING
      const uint32_t t_i0 = (uint32_t)clock();
#endif
      if (f_iss < fb) issue_next(); else cp_async_commit();
#ifdef OC_PROBE_TIMING
      if (lane == 0 && blockIdx.x == 0 && p.score && i < 16) {
        uint32_t* pr = reinterpret_cast<uint32_t*>(p.score) + (warp * 16 + i) * 4;
        pr[0] = t_w0;
        pr[1] = t_w1;
        pr[2] = t_i0;
        pr[3] = (uint32_t)clock();
      }
#endif
    }
    if (ATTN && seg_unit >= 0 && seg_kept && lane == 0) atomicAdd(p.cnt_unit + seg_unit, (uint32_t)seg_kept);
  }
  if (p.stats && lane == 0 && kept_stat) atomicAdd(p.stats, (uint32_t)kept_stat);
#ifdef OC_PROBE_SPAN
  if (lane == 0 && p.score) {
    uint64_t span_t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(span_t1));
    reinterpret_cast<uint64_t*>(p.score)[2 * wg] = span_t0;
    reinterpret_cast<uint64_t*>(p.score)[2 * wg + 1] = span_t1;
  }
#endif
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
    for (int i = 0; i < NSLOT; ++i) {
      if (i < nB) issue_next_v(); else cp_async_commit();
    }

    float m_run[GC], l_part[GC];
    float2 acc[TC ? 1 : GC][D2];
    // tensor-core path: this lane's query g8 (m, partial l) and O^T fragments
    float m_mine = -1e9f, l_mine = 0.f;
    float tacc[TC ? HD / 16 : 1][4];
    int cur_unit = -1;
    auto reset_state = [&]() {
      if constexpr (TC) {
        m_mine = -1e9f;
        l_mine = 0.f;
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j) tacc[mt][j] = 0.f;
        return;
      }
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
      const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
      const int gvalid = (p.group - chunk * GC) < GC ? (p.group - chunk * GC) : GC;
      const int hq0 = kvh * p.group + chunk * GC;
      const int64_t R0 = kp[u], R1 = (int64_t)kp[u + 1] - 1;
      const int64_t w0 = range_owner(R0, Kt, WB), w1 = range_owner(R1, Kt, WB);
      const bool direct = (w0 == w1);
      const int64_t slot = direct ? 0 : partial_slot(wg, R0, Kt, WB);
      // put(query, dim, m, l, acc): write the merged state of one output element
      auto put = [&](int qq, int d, float m, float l, float a) {
        if (direct) {
          if (qq < gvalid) emit(p, seq, hq0 + qq, d, m, l, a);
        } else if (qq < GC) {
          part[(slot * GC + qq) * PST + d] = a;
        }
      };
      if constexpr (TC) {
        float lq = l_mine + __shfl_xor_sync(0xffffffffu, l_mine, 1);
        lq += __shfl_xor_sync(0xffffffffu, lq, 2);
        const int qa = 2 * t4, qb = 2 * t4 + 1;
        const float ma = __shfl_sync(0xffffffffu, m_mine, (8 * t4) & 31);
        const float mb = __shfl_sync(0xffffffffu, m_mine, (8 * t4 + 4) & 31);
        const float la = __shfl_sync(0xffffffffu, lq, (8 * t4) & 31);
        const float lb = __shfl_sync(0xffffffffu, lq, (8 * t4 + 4) & 31);
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt) {
          put(qa, 16 * mt + g8, ma, la, tacc[mt][0]);
          put(qb, 16 * mt + g8, mb, lb, tacc[mt][1]);
          put(qa, 16 * mt + g8 + 8, ma, la, tacc[mt][2]);
          put(qb, 16 * mt + g8 + 8, mb, lb, tacc[mt][3]);
        }
        if (!direct && t4 == 0 && g8 < GC)
          *reinterpret_cast<float2*>(part + (slot * GC + g8) * PST + HD) = make_float2(m_mine, lq);
      } else {
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
        if (rg == 0)
#pragma unroll
          for (int g = 0; g < GC; ++g) {
#pragma unroll
            for (int d = 0; d < D2; ++d) {
              put(g, c * DPT + 2 * d, m_run[g], lsum[g], acc[g][d].x);
              put(g, c * DPT + 2 * d + 1, m_run[g], lsum[g], acc[g][d].y);
            }
            if (!direct && c == 0)
              *reinterpret_cast<float2*>(part + (slot * GC + g) * PST + HD) = make_float2(m_run[g], lsum[g]);
          }
      }
      if (direct) return;
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
      if constexpr (TC) {
        // this lane's query g8: logits of tokens 16ks + 2t4 + {0,1,8,9}
        float lv[4][4];
        float lmax = -INFINITY;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const float2 x = g8 < GC ? *reinterpret_cast<const float2*>(lgs + g8 * 64 + 16 * ks + 2 * t4)
                                   : make_float2(-INFINITY, -INFINITY);
          const float2 y = g8 < GC ? *reinterpret_cast<const float2*>(lgs + g8 * 64 + 16 * ks + 2 * t4 + 8)
                                   : make_float2(-INFINITY, -INFINITY);
          lv[ks][0] = x.x; lv[ks][1] = x.y; lv[ks][2] = y.x; lv[ks][3] = y.y;
          lmax = fmaxf(lmax, fmaxf(fmaxf(x.x, x.y), fmaxf(y.x, y.y)));
        }
        lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, 1));
        lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, 2));
        const float nm = fmaxf(m_mine, lmax);
        const float alpha = exp2f(m_mine - nm);
        m_mine = nm;
        // P split into a 16-bit head and tail so that P V keeps ~16 significant bits
        uint32_t bh[4][2], bl[4][2];
        float psum = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          float pr[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            pr[j] = g8 < GC ? exp2f(lv[ks][j] - nm) : 0.f;
            psum += pr[j];
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if constexpr (KBF16) {
              const __nv_bfloat162 hi = __floats2bfloat162_rn(pr[2 * h], pr[2 * h + 1]);
              const float2 hf = __bfloat1622float2(hi);
              const __nv_bfloat162 lo = __floats2bfloat162_rn(pr[2 * h] - hf.x, pr[2 * h + 1] - hf.y);
              bh[ks][h] = *reinterpret_cast<const uint32_t*>(&hi);
              bl[ks][h] = *reinterpret_cast<const uint32_t*>(&lo);
            } else {
              const __half2 hi = __floats2half2_rn(pr[2 * h], pr[2 * h + 1]);
              const float2 hf = __half22float2(hi);
              const __half2 lo = __floats2half2_rn(pr[2 * h] - hf.x, pr[2 * h + 1] - hf.y);
              bh[ks][h] = *reinterpret_cast<const uint32_t*>(&hi);
              bl[ks][h] = *reinterpret_cast<const uint32_t*>(&lo);
            }
          }
        }
        l_mine = fmaf(l_mine, alpha, psum);
        // rescale the O^T columns (queries 2t4, 2t4+1) by their alphas
        const float a0 = __shfl_sync(0xffffffffu, alpha, (8 * t4) & 31);
        const float a1 = __shfl_sync(0xffffffffu, alpha, (8 * t4 + 4) & 31);
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt) {
          tacc[mt][0] *= a0; tacc[mt][1] *= a1; tacc[mt][2] *= a0; tacc[mt][3] *= a1;
        }
        // O^T (dims x queries) += V^T (dims x tokens) * P (tokens x queries)
        const uint32_t base = smem_u32(ts);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
          for (int mt = 0; mt < HD / 16; ++mt) {
            uint32_t a4[4];
            ldsm_x4_t(tc_addr(base, 16 * ks + (lane & 7) + ((lane >> 4) & 1) * 8, 16 * mt + ((lane >> 3) & 1) * 8,
                              CF::ROWV), a4);
            mma16816<KBF16>(tacc[mt], a4, bh[ks][0], bh[ks][1]);
            mma16816<KBF16>(tacc[mt], a4, bl[ks][0], bl[ks][1]);
          }
      } else {
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
#pragma unroll kUnrollPV
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
      }
      __syncwarp();
      ++item;
      if (j_iss < nB) issue_next_v(); else cp_async_commit();
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

template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT, bool TC>
cudaError_t launch_decode(const DecodeParams& p, int num_sms, cudaStream_t stream) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT>;
  auto kern = decode_kernel<KT, VT, HD, GC, ATTN, NSLOT, TC>;
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
