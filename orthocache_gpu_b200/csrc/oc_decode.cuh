// Fused spectral-eviction decode attention for B200 (sm_100a).
//
// One kernel template serves every variant of the reference's hot path
// (j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/):
//   * V1 / V2 zeta-gated split-K decode ........ fused_eviction.py:84-373
//   * V3 Cauchy-Schwarz GQA gate ............... gqa_eviction.py:286-495
//   * paged KV (block-table gather) ............ paged_eviction.py:56-237
//   * mask / zeta scoring only ................. fwht_fused_prototype.py:102-192
//
// Design: one persistent CTA per SM.  On the tensor-core path a team of
// HD/64 warps shares each tile (one 64-column panel per warp); otherwise a
// team is one warp.  Every warp has its own shared-memory ring of tile slots
// filled by TMA (one mbarrier per slot, consumed in order), so the per-tile
// path has no CTA-wide or grid-wide barrier; a team's warps meet only at a
// named barrier to add their panels' band energies and logits.
//
//   The tiles of all units (sequence, kv head, query chunk) are flattened
//   (oc_plan.h) and split into equal contiguous ranges, one per team; inside a
//   unit the order is the reference's interleaved split order, so a range
//   samples the whole sequence.  A team scores each 64-token K tile; for a
//   retained tile it computes the query logits (fp32, log2 domain) into the
//   slot's logit area and reuses the slot for the tile's V, which is consumed
//   after the copies already in flight.  An evicted tile costs one K read;
//   its V is never read.  A unit's online-softmax state is written once its K
//   tiles in the range are gated and no V copy of it is pending: directly
//   when the range holds the whole unit, else as a partial state that
//   merge_kernel (a programmatic dependent launch) combines by log-sum-exp.
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

#include <cuda.h>
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
//   GATE_LIST:      no gate; each (sequence, kv head) decodes the tiles of its
//                   list (tile_list / list_count), e.g. the tiles a cached-norm
//                   gate retained, so evicted tiles cost no K or V read at all
enum : int { GATE_ZETA_ATTN = 0, GATE_ZETA_MASK = 1, GATE_CS = 2, GATE_LIST = 3 };
enum : int { LAYOUT_LINEAR = 0, LAYOUT_PAGED = 1 };
enum : uint32_t { ST_TIMEOUT = 1u, ST_BAD_PAGE = 2u, ST_BAD_SEQLEN = 4u };

constexpr uint32_t kWaitLimit = 1u << 22;
#ifndef OC_TILES_PER_TEAM
#define OC_TILES_PER_TEAM 1
#endif
constexpr int kTilesPerTeam = OC_TILES_PER_TEAM;  // grid sizing for small problems

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
// Width in columns of a warp's panel on the tensor-core path: 64 (128-byte
// rows, 128-byte TMA swizzle) or 32 (64-byte rows, 64-byte swizzle; twice the
// warps share a tile).
#ifndef OC_TC_PANEL
#define OC_TC_PANEL 64
#endif
constexpr int kTcPanel = OC_TC_PANEL;
static_assert(kTcPanel == 64 || kTcPanel == 32, "tensor-core panel width");
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
  int box_rows;  // tokens per TMA box: 64, or the page size when pages are smaller
  int tm_pos_k[3], tm_pos_v[3];  // tensor-map dimension of the token / kv-head / outer index
  int num_seqs, num_kv_heads, group, num_tiles, num_splits;
  int gate;
  float thr;
  float scale_log2;  // log2(e)/sqrt(head_dim)
  void* out;
  int out_dtype;
  int64_t out_seq_stride, out_head_stride;
  int8_t* mask;       // (num_seqs, num_kv_heads, num_tiles), nullable
  float* score;       // same shape: zeta or Cauchy-Schwarz bound, nullable
  uint32_t* stats;    // [0] = retained tiles of the call (written by merge_kernel), nullable
  int stats_add;      // 1: add this launch's count to stats[0] (later launches of one call)
  uint32_t* status;   // error bits (sticky OR), non-null
  // workspace (attention only)
  int* tile_prefix;    // tiles of units [0, u): written by CTA 0 for merge_kernel (units + 1 ints)
  int* team_kept;      // retained tiles gated by each team of the grid (one int per team)
  float* part;         // partial states [2 * teams][GC][P][HD/P + 4]: acc, m, l
  // shard mode (nullable): write the merged partial state (m, l, unnormalised
  // acc) of each query head instead of the normalised output
  float* sh_m;
  float* sh_l;
  float* sh_acc;
  // float8 keys of the paged path are de-quantised as the reference does
  // (paged_eviction.py:355-357: k_cache.to(q.dtype) * k_scale): every key
  // element becomes round_to(k_deq_dtype, float(k) * k_deq_scale) before the
  // gate and the logits.  k_deq_dtype < 0: keys are used as stored.
  int k_deq_dtype;
  float k_deq_scale;
  // GATE_LIST: tiles of (seq, kv head) g are tile_list[g*list_stride + k], k < list_count[g]
  const int* tile_list;
  const int* list_count;
  int64_t list_stride;
  // diagnostics (written only in builds with OC_TRACE defined): per team 16
  // timestamps / counters, then 3 per merge block; see oc_debug_set_trace
  unsigned long long* trace;
};

__device__ __forceinline__ unsigned long long oc_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

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

// De-quantisation of float8 keys into the query dtype (see DecodeParams::k_deq_dtype).
template <typename KT, int N>
__device__ __forceinline__ void k_dequant(const DecodeParams& p, float2 (&f)[N]) {
  if constexpr (std::is_same<KT, __nv_fp8_e4m3>::value) {
    if (p.k_deq_dtype >= 0) {
      const float s = p.k_deq_scale;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float2 x = make_float2(f[i].x * s, f[i].y * s);
        if (p.k_deq_dtype == DT_F16) x = __half22float2(__floats2half2_rn(x.x, x.y));
        else if (p.k_deq_dtype == DT_BF16) x = __bfloat1622float2(__floats2bfloat162_rn(x.x, x.y));
        f[i] = x;
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float2 warp_sum2(float2 x) {  // two independent butterflies
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    x.x += __shfl_xor_sync(0xffffffffu, x.x, o);
    x.y += __shfl_xor_sync(0xffffffffu, x.y, o);
  }
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

// ---------------------------------------------------------------- config
template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT, bool TC>
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
  // Tensor-core path: a team of P = HD/64 warps shares each tile, one
  // 64-column panel (HDL columns) per warp; otherwise P = 1.
  static constexpr int P = TC ? HD / kTcPanel : 1;
  static constexpr int HDL = HD / P;
  static constexpr int SLOT = 64 * ROWMAX / P;  // a multiple of 1024: swizzle atoms stay aligned
  static constexpr int RING = 208 * 1024;
  static constexpr int NW0 = RING / (NSLOT * (SLOT + LGB));
  static constexpr int NWC = NW0 > kMaxWarpsPerCta ? kMaxWarpsPerCta : NW0;
  static constexpr int NW = NWC < P ? P : NWC / P * P;  // whole teams
  static constexpr int NT = NW * 32;
  static constexpr int MAXU = 2048;  // units per launch (the host batches larger problems)
  static constexpr int MAXT = 1280;  // teams per grid (partial-state slots of the workspace)
  static constexpr int OFF_LGS = NW * NSLOT * SLOT;         // logits of slot s: [NW][NSLOT][GC*64] floats
  static constexpr int OFF_BAR = OFF_LGS + NW * NSLOT * LGB;  // full barrier of each slot
  static constexpr int OFF_XCH = OFF_BAR + 8 * NW * NSLOT;    // band energies exchanged in a team: [NW/P][2][P] float2
  static constexpr int OFF_STG = OFF_XCH + 16 * NW;              // finalize staging, 64 floats a warp (8-byte aligned)
  static constexpr int OFF_TP = OFF_STG + 256 * NW;
  static constexpr int OFF_MISC = OFF_TP + 4 * (MAXU + 1);
  static constexpr int SMEM = (OFF_MISC + 4 * 32 + 127) / 128 * 128 + 1024;  // + base alignment slack
  static_assert(C >= 1 && C <= 32 && (C & (C - 1)) == 0, "K row bytes must be a power of two in 16..512");
  static_assert(D2 >= 2 && (VCB % 16) == 0, "vector widths");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Block-wide inclusive scan of a[1..n] in place, a[0] = 0; tmp holds one int per warp.
// Each thread scans a contiguous chunk; chunk totals are scanned with warp shuffles.
__device__ __noinline__ static void block_scan(int* a, int n, int* tmp) {
  __syncthreads();
  const int nt = blockDim.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (n + nt - 1) / nt;
  const int lo = 1 + tid * per, hi = min(n + 1, lo + per);
  int run = 0;
  for (int i = lo; i < hi; ++i) run += a[i];
  int inc = run;  // inclusive scan of the chunk totals inside the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) tmp[wid] = inc;
  __syncthreads();
  int base = inc - run;
  for (int w = 0; w < wid; ++w) base += tmp[w];
  for (int i = lo; i < hi; ++i) {
    base += a[i];
    a[i] = base;
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
__global__ void __launch_bounds__(Cfg<KT, VT, HD, GC, ATTN, NSLOT, TC>::NT, 1)
    decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT, TC>;
  constexpr int C = CF::C, RG = CF::RG, RPL = CF::RPL, PAIRS = CF::PAIRS, DPT = CF::DPT, D2 = CF::D2;
  constexpr int RGE = CF::RGE, NRES = CF::NRES, NW = CF::NW, SLOT = CF::SLOT;
  constexpr int P = CF::P, HDL = CF::HDL;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // 1024-byte aligned base: the TMA 128-byte swizzle repeats every 1024 bytes
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#ifdef OC_TRACE
  const unsigned long long tr_t0 = oc_clock();
  unsigned long long tr_t1 = 0, tr_t2 = 0, tr_a = 0, tr_b = 0, tr_x[4] = {0, 0, 0, 0};
  int tr_nk = 0, tr_nv = 0;
  unsigned long long tr_wait = 0, tr_sync = 0, tr_polls = 0;
  long long tr_sec[6] = {0, 0, 0, 0, 0, 0};  // SM cycles: gate, logits, V step, issue, finalize, loop
#define OC_TR_BEGIN(v) const long long v = clock64()
#define OC_TR_END(i, v) tr_sec[i] += clock64() - (v)
#else
#define OC_TR_BEGIN(v)
#define OC_TR_END(i, v)
#endif
  const int c = lane % C, rg = lane / C;
  static_assert(!TC || (CF::KB == 2 && CF::VB == 2 && HD >= 64 && GC <= 8), "tensor-core path");
  constexpr bool KBF16 = TC && (sizeof(KT) == 2) && !std::is_same<KT, __half>::value;
  const int g8 = lane >> 2, t4 = lane & 3;  // mma fragment coordinates
  // team of P warps (one 64-column panel each on the tensor-core path); work is assigned per team
  const int team = warp / P, panel = warp % P;
  const int64_t W = (int64_t)gridDim.x * (NW / P);        // teams in the grid
  const int64_t wg = (int64_t)blockIdx.x * (NW / P) + team;  // this warp's team
  auto team_sync = [&]() {
#ifdef OC_TRACE
    const unsigned long long c0 = oc_clock();
#endif
    if constexpr (P > 1) asm volatile("bar.sync %0, %1;" ::"r"(team + 1), "r"(32 * P) : "memory");
#ifdef OC_TRACE
    tr_sync += oc_clock() - c0;
#endif
  };
  const int nchunks = (p.group + GC - 1) / GC;
  const int U = p.num_seqs * p.num_kv_heads * nchunks;
  const int S = p.num_splits;

  int* tp = reinterpret_cast<int*>(smem + CF::OFF_TP);
  int* scan_tmp = reinterpret_cast<int*>(smem + CF::OFF_MISC);
  unsigned char* ring = smem + warp * NSLOT * SLOT;
  float* lgs_all = reinterpret_cast<float*>(smem + CF::OFF_LGS);  // [NW][NSLOT][GC*64]
  float* lgs_base = lgs_all + warp * NSLOT * (CF::LGB / 4);
  float2* xch = reinterpret_cast<float2*>(smem + CF::OFF_XCH) + team * 2 * P;
  float* stg = reinterpret_cast<float*>(smem + CF::OFF_STG) + warp * 64;  // finalize staging
  const uint32_t bar0 = smem_u32(smem + CF::OFF_BAR) + 8u * warp * NSLOT;  // this warp's slot barriers
  if (tid == 0) {  // fetch the copy descriptors while the prologue runs
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
    if (ATTN) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmV) : "memory");
  }
  if (lane < NSLOT) mbar_init(bar0 + 8u * lane, 1);
  mbar_init_fence();
  __syncwarp();

  // Every launch is a programmatic dependent of the kernel before it on the
  // stream (in LIST mode the gate kernel that wrote the lists): the set-up
  // that reads no global memory overlaps that kernel's tail.  Without
  // per-sequence lengths or tile lists that is everything up to the first
  // read of q (the tile prefix and the team's range come from the
  // parameters); otherwise the prefix reads them, so the wait comes first.
  const bool late_wait = p.seq_lens == nullptr && p.list_count == nullptr;
  if (!late_wait) asm volatile("griddepcontrol.wait;" ::: "memory");
  // ---- tiles per unit, prefix in shared memory.  Without per-sequence
  // lengths or tile lists every unit has num_tiles tiles: each warp writes
  // the whole prefix itself (every warp writes the same values), so no block
  // barrier and no scan delay the first copies.
  if (p.seq_lens == nullptr && p.list_count == nullptr) {
    for (int u = lane; u <= U; u += 32) tp[u] = u * p.num_tiles;
    __syncwarp();
#ifdef OC_TRACE
    tr_a = oc_clock();
#endif
  } else {
    for (int u = tid; u < U; u += blockDim.x) {
      int T = p.num_tiles;
      if (p.seq_lens != nullptr) {
        const int L = p.seq_lens[u / (p.num_kv_heads * nchunks)];
        if ((L < 0 || (L & 63) || L > p.num_tiles * 64) && blockIdx.x == 0) atomicOr(p.status, ST_BAD_SEQLEN);
        const int lt = L < 0 ? 0 : (L >> 6);
        T = lt < T ? lt : T;
      }
      if (p.list_count != nullptr) {
        const int c = p.list_count[u / nchunks];
        T = c < 0 ? 0 : (c < T ? c : T);
      }
      tp[u + 1] = T;
    }
#ifdef OC_TRACE
    __syncwarp();
    tr_a = oc_clock();
#endif
    if (U <= 32 * 32) {  // one warp scans (up to 32 values a lane)
      __syncthreads();
      if (warp == 0) {
        const int per = (U + 31) / 32, lo = 1 + lane * per, hi = min(U + 1, lo + per);
        int run = 0;
        for (int i = lo; i < hi; ++i) run += tp[i];
        int inc = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += y;
        }
        int base = inc - run;
        for (int i = lo; i < hi; ++i) {
          base += tp[i];
          tp[i] = base;
        }
        if (lane == 0) tp[0] = 0;
      }
      __syncthreads();
    } else {
      block_scan(tp, U, scan_tmp);
    }
  }
  const int64_t N = tp[U];
#ifdef OC_TRACE
  tr_x[0] = oc_clock();
#endif
  // Team wg owns the flattened K tiles [fa, fb) (see the single pass below)
  const int64_t WE = (N < W) ? (N > 0 ? N : 1) : W;  // warps with a tile range
#ifdef OC_TRACE
  tr_x[1] = oc_clock();
#endif
  const bool active = wg < WE;
  // flattened tile indices fit in 32 bits (at most 2048 units of 2^20 tiles): the loop uses int
  const int fa = active ? (int)range_lo(wg, N, WE) : 0, fb = active ? (int)range_lo(wg + 1, N, WE) : 0;
  const uint64_t pol = policy_evict_first();

  auto unit_seq = [&](int u) { return u / (p.num_kv_heads * nchunks); };
  auto unit_kvh = [&](int u) { return (u / nchunks) % p.num_kv_heads; };
  auto unit_chunk = [&](int u) { return u % nchunks; };
  auto tile_of = [&](int u, int64_t f) { return split_major_tile((int)(f - tp[u]), tp[u + 1] - tp[u], S); };

  // smem address of (token, dim) of a 16-bit tile on the tensor-core path:
  // 64-column panels of 64 tokens x 128 bytes, the 16-byte chunks of a row
  // XORed with (token & 7) by the TMA 128-byte swizzle, so ldmatrix reads of
  // 8 rows hit 8 distinct bank groups.
  //   tc_addr(tok, dim) = base + tok * 128 + ((((dim * 2) >> 4) ^ (tok & 7)) << 4)  (dim < 64)
  // Per-lane parts of the ldmatrix addresses (x = lane & 7, b3 / b4 = lane bits 3 / 4):
  // every row a lane addresses has (row & 7) == x, so the swizzled chunk of
  // column 16 c + 8 b is ((2 c + b) ^ x).
  // With 32-column panels rows are 64 bytes and the 64-byte swizzle XORs the
  // chunk (0..3) with (token >> 1) & 3, which is (x >> 1) & 3 for every row a
  // lane addresses.
  constexpr uint32_t kRowB = 2u * HDL;  // bytes of a panel row
  const uint32_t kSwz = HDL == 64 ? (uint32_t)(lane & 7) : (uint32_t)((lane & 7) >> 1);
  uint32_t ch3[TC ? HDL / 16 : 1], ch4[TC ? HDL / 16 : 1];
  uint32_t offG = 0, offL = 0, offV = 0;
  if constexpr (TC) {
    const uint32_t x = lane & 7, b3 = (lane >> 3) & 1, b4 = (lane >> 4) & 1;
#pragma unroll
    for (int c2 = 0; c2 < HDL / 16; ++c2) {
      ch3[c2] = ((2u * c2 + b3) ^ kSwz) << 4;
      ch4[c2] = ((2u * c2 + b4) ^ kSwz) << 4;
    }
    offG = (x + 32u * b4) * kRowB;  // gate: tokens 8 s4 + x (+32), columns 16 np + 8 b3
    offL = (x + 8u * b3) * kRowB;   // logits: tokens 16 mt + x + 8 b3, columns 16 ks + 8 b4
    offV = (x + 8u * b4) * kRowB;   // P V: tokens 16 ks + x + 8 b4, columns 16 mt + 8 b3
  }

  // TMA copy of tile `tile` of unit u (K or V) into ring slot s: one box per
  // page run (of this warp's 64-column panel on the tensor-core path), all
  // completing on the slot's barrier.
  // The slot was only read (generic proxy) since its last copy, so the next
  // copy needs no proxy fence: __syncwarp orders the lanes' reads before it.
  // Paged layout: block-table windows, one for the K copy cursor and one for
  // the V copy cursor.  Lane i holds entry base + i of sequence wseq, loaded
  // by one coalesced warp load; a tile's page ids are then read with a
  // shuffle instead of a dependent global load per copy.  Tiles of a team are
  // consecutive inside a unit (the paged path runs with one split), so a
  // window of 32 pages serves 512 / 64 * page_size tokens.
  int win_seq[2] = {-1, -1}, win_base[2] = {0, 0};
  int win_val[2] = {0, 0};
  const int max_pages = p.layout == LAYOUT_PAGED ? ((p.num_tiles * 64 + (1 << p.block_shift) - 1) >> p.block_shift) : 0;
  auto issue = [&](uint32_t s, int seq, int kvh, int tile, bool isv) {
    const uint32_t fbar = bar0 + 8u * s;
    const uint32_t dst = smem_u32(ring + s * SLOT);
    const int row = isv ? CF::ROWV : CF::ROWK;
    const void* tm = isv ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
    const int pt = isv ? p.tm_pos_v[0] : p.tm_pos_k[0];  // tensor-map dimension of the token index
    const int ph = isv ? p.tm_pos_v[1] : p.tm_pos_k[1];  // ... of the kv-head index
    // coordinate of tensor-map dimension d (1..3)
    auto crd = [&](int d, int tok, int kvh_, int outer) { return d == pt ? tok : (d == ph ? kvh_ : outer); };
    __syncwarp();
    if (p.layout == LAYOUT_LINEAR) {  // one box of 64 rows
      if (lane == 0) {
        mbar_arrive_expect_tx(fbar, 64u * row / P);
        tma_load_4d(dst, tm, panel * HDL, crd(1, tile * 64, kvh, seq), crd(2, tile * 64, kvh, seq),
                    crd(3, tile * 64, kvh, seq), fbar, pol);
      }
      return;
    }
    if (lane == 0) mbar_arrive_expect_tx(fbar, 64u * row / P);
    __syncwarp();
    const int RB = p.box_rows;
    const int nruns = 64 / RB;
    if (nruns <= 32) {
      const int w = isv ? 1 : 0;
      const int first = (tile * 64) >> p.block_shift, last = (tile * 64 + 63) >> p.block_shift;
      if (seq != win_seq[w] || first < win_base[w] || last >= win_base[w] + 32) {  // warp-uniform
        win_seq[w] = seq;
        win_base[w] = first;
        const int e = first + lane;
        win_val[w] = e < max_pages ? p.block_tables[(int64_t)seq * p.bt_seq_stride + e] : 0;
      }
      const int t = tile * 64 + (lane < nruns ? lane : 0) * RB;
      int pb = __shfl_sync(0xffffffffu, win_val[w], (t >> p.block_shift) - win_base[w]);
      if (lane < nruns) {
        if (pb < 0 || pb >= p.num_blocks) {
          atomicOr(p.status, ST_BAD_PAGE);
          pb = 0;
        }
        const int tk = t & ((1 << p.block_shift) - 1);
        tma_load_4d(dst + (uint32_t)(lane * RB * (row / P)), tm, panel * HDL, crd(1, tk, kvh, pb),
                    crd(2, tk, kvh, pb), crd(3, tk, kvh, pb), fbar, pol);
      }
      return;
    }
    for (int run = lane; run < nruns; run += 32) {
      const int t = tile * 64 + run * RB;
      int pb = p.block_tables[(int64_t)seq * p.bt_seq_stride + (t >> p.block_shift)];
      if (pb < 0 || pb >= p.num_blocks) {
        atomicOr(p.status, ST_BAD_PAGE);
        pb = 0;
      }
      const int tk = t & ((1 << p.block_shift) - 1);
      tma_load_4d(dst + (uint32_t)(run * RB * (row / P)), tm, panel * HDL, crd(1, tk, kvh, pb), crd(2, tk, kvh, pb),
                  crd(3, tk, kvh, pb), fbar, pol);
    }
  };

  // Wait for the copy in slot s (bounded; a timeout sets the status bit).
  uint32_t phases = 0;  // bit s: parity of slot s's next completion
  auto wait_slot = [&](uint32_t s) {
#ifdef OC_TRACE
    const unsigned long long c0 = oc_clock();
#endif
#ifdef OC_TRACE
    {
      uint32_t i = 0;
      while (i < kWaitLimit && !mbar_try_wait(bar0 + 8u * s, (phases >> s) & 1u)) ++i;
      tr_polls += i + 1;
      if (i == kWaitLimit && lane == 0) atomicOr(p.status, ST_TIMEOUT);
    }
#else
    if (!mbar_wait_bounded(bar0 + 8u * s, (phases >> s) & 1u, kWaitLimit) && lane == 0)
      atomicOr(p.status, ST_TIMEOUT);
#endif
#ifdef OC_TRACE
    tr_wait += oc_clock() - c0;
#endif
    phases ^= 1u << s;
    __syncwarp();
    return ring + s * SLOT;
  };

  // ---- the first copies go out before the rest of the set-up
  float2 qv[TC ? 1 : GC][D2];
  uint32_t qf[TC ? HDL / 16 : 1][2];  // q (this warp's panel) as mma B fragments (dims x queries), raw 16-bit
  int q_unit = -1;
  uint32_t qf_pf[TC ? HDL / 16 : 1][2];  // prefetched fragments of unit pf_unit
  int pf_unit = -1;
  // q rows of a unit's query chunk (this warp's panel) as raw 16-bit mma B fragments
  // The loads are issued unconditionally (lanes without a query read the
  // chunk's first head) and nothing consumes them here, so the warp does not
  // wait for them: qf_apply masks the lanes without a query when the
  // fragments are first used.  q rows are 4-byte aligned (checked on the host).
  auto load_qf = [&](int seq, int kvh, int chunk, uint32_t (&dst)[TC ? HDL / 16 : 1][2], bool& ok) {
    if constexpr (TC) {
      const int hq = chunk * GC + g8;
      ok = g8 < GC && hq < p.group;
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          static_cast<const uint16_t*>(p.q) + (int64_t)seq * p.q_seq_stride +
          (int64_t)(kvh * p.group + (ok ? hq : chunk * GC)) * p.q_head_stride + panel * HDL);
#pragma unroll
      for (int ks = 0; ks < HDL / 16; ++ks) {
        dst[ks][0] = qrow[8 * ks + t4];
        dst[ks][1] = qrow[8 * ks + t4 + 4];
      }
    }
  };
  bool qok_pf = false;
  auto qf_apply = [&](const uint32_t (&src)[TC ? HDL / 16 : 1][2], bool ok) {
#pragma unroll
    for (int ks = 0; ks < (TC ? HDL / 16 : 1); ++ks) {
      qf[ks][0] = ok ? src[ks][0] : 0u;
      qf[ks][1] = ok ? src[ks][1] : 0u;
    }
  };

  // descriptor of ring slot `lane` (lanes < NSLOT): flattened tile (-1: empty),
  // V copy flag, unit and tile index
  //   dsc_a = 2 * (f - fa) + (V copy), or -1 for an empty slot; dsc_b = (unit << 20) | tile
  int dsc_a = -1, dsc_b = 0;
#ifdef OC_TRACE
  tr_x[3] = oc_clock();
#endif
  const int u_first = (fb > fa) ? upper_index(tp, U, fa) : 0;
  int u_iss = u_first, seq_iss = 0, kvh_iss = 0;
  int u_end_iss = 0;  // first flattened tile after unit u_iss
  int f_iss = fa;
  SplitIter it_iss;
  // GATE_LIST: list entry of the next tile to issue, loaded one issue ahead
  int list_pf = 0;
  auto list_load = [&](int u, int f) {
    return p.tile_list[(int64_t)(u / nchunks) * p.list_stride + (f - tp[u])];
  };
  auto enter_unit = [&](int u, int f) {  // issue cursor enters unit u at flattened tile f
    u_iss = u;
    u_end_iss = tp[u + 1];
    seq_iss = unit_seq(u);
    kvh_iss = unit_kvh(u);
    if constexpr (ATTN && TC) {
      load_qf(seq_iss, kvh_iss, unit_chunk(u), qf_pf, qok_pf);
      pf_unit = u;
    }
    it_iss.init((int)(f - tp[u]), tp[u + 1] - tp[u], S);
    if (p.tile_list != nullptr) list_pf = list_load(u, f);
  };
#ifdef OC_TRACE
  tr_b = oc_clock();
#endif
  if (late_wait) asm volatile("griddepcontrol.wait;" ::: "memory");
  if (fb > fa) enter_unit(u_first, fa);
#ifdef OC_TRACE
  unsigned long long tr_c = oc_clock(), tr_d = 0;
#endif
  // LIST mode: every tile is retained, so a tile's V copy is issued into the
  // slot right after its K copy (both in flight at once); the V item reads
  // the logits its K item left in the preceding slot's logit area.
#ifndef OC_LIST_PAIRED
#define OC_LIST_PAIRED 0  // measured slower (192 vs 209 us at the V3 shapes); kept as a build option
#endif
  const bool paired = OC_LIST_PAIRED && ATTN && p.tile_list != nullptr;
  int pend_v = 0, pv_seq = 0, pv_kvh = 0, pv_tile = 0, pv_da = 0, pv_u = 0;
  auto issue_next = [&](uint32_t s) {
    if (paired && pend_v) {
      issue(s, pv_seq, pv_kvh, pv_tile, true);
      if (lane == (int)s) {
        dsc_a = pv_da | 1;
        dsc_b = (pv_u << 20) | pv_tile;
      }
      pend_v = 0;
      return;
    }
    if (f_iss < fb) {
      if (f_iss >= u_end_iss) {
        int u = u_iss + 1;
        while (f_iss >= tp[u + 1]) ++u;
        enter_unit(u, f_iss);
      }
      const int tile = p.tile_list != nullptr ? list_pf : it_iss.tile();
      issue(s, seq_iss, kvh_iss, tile, false);
      if (lane == (int)s) {
        dsc_a = 2 * (int)(f_iss - fa);
        dsc_b = (u_iss << 20) | tile;
      }
      if (paired) {
        pend_v = 1;
        pv_seq = seq_iss;
        pv_kvh = kvh_iss;
        pv_tile = tile;
        pv_da = 2 * (int)(f_iss - fa);
        pv_u = u_iss;
      }
      it_iss.next();
      ++f_iss;
      if (p.tile_list != nullptr && f_iss < u_end_iss && f_iss < fb) list_pf = list_load(u_iss, f_iss);
    } else if (lane == (int)s) {
      dsc_a = -1;
    }
  };
  for (uint32_t s = 0; s < NSLOT; ++s) {
    issue_next(s);
#ifdef OC_TRACE
    if (s == 0) tr_d = oc_clock();
#endif
  }
#ifdef OC_TRACE
  tr_t1 = oc_clock();
#endif

  if (ATTN && blockIdx.x == 0)
    for (int u = tid; u <= U; u += blockDim.x) p.tile_prefix[u] = tp[u];

  float qmax = 0.f;  // max_g |q_g| of the current unit (Cauchy-Schwarz gate)
  uint32_t ktiles = 0;  // K tiles gated (selects the team's exchange buffer)
  // ---- tensor-core gate constants.  The gate runs with the K tile as the A
  // operand (A = K^T: 16 head-dim columns x 16 tokens) and a constant B:
  // each k-step takes tokens {t0..t0+7} and {t0+32..t0+39}, so
  //   B_low[k][n]  = W[n+1][k & 7]      (rows 1..7 of the 64-point natural-order
  //                                      Walsh matrix depend only on token bits 0..2)
  //   B_diff[k][n] = +1 if k == n, -1 if k == n + 8
  // give, per k-step, 16 columns x (W K)_{1..7} partial sums and the 8
  // differences K[t0+n] - K[t0+32+n].  Four k-steps (t0 = 0, 8, 16, 24) cover
  // the tile: 8 MMAs per 16 columns.
  uint32_t bLow = 0u, bDiff = 0u, bNeg = 0u;
  if constexpr (TC) {
    const uint32_t P8 = KBF16 ? 0x3E00u : 0x3000u, N8 = KBF16 ? 0xBE00u : 0xB000u;  // +-1/8
    const uint32_t ONE = KBF16 ? 0x3F80u : 0x3C00u, MONE = KBF16 ? 0xBF80u : 0xBC00u;
    auto w = [&](int r, int tk) -> uint32_t {
      if (r < 1 || r > 7) return 0u;  // row 0 (DC) and rows >= 8 do not enter E_low
      return (__popc(r & tk) & 1) ? N8 : P8;
    };
    // B fragment: this lane holds B[2t4][g8], B[2t4+1][g8] (register 0) and rows +8 (register 1)
    bLow = w(g8 + 1, 2 * t4) | (w(g8 + 1, 2 * t4 + 1) << 16);  // same for rows k+8 (same low bits)
    bDiff = (g8 == 2 * t4 ? ONE : 0u) | ((g8 == 2 * t4 + 1 ? ONE : 0u) << 16);
    bNeg = (g8 == 2 * t4 ? MONE : 0u) | ((g8 == 2 * t4 + 1 ? MONE : 0u) << 16);
  }
  // E_low = sum (W K)[1..7]^2 and E_high = 1/2 sum (K[t]-K[t+32])^2
  auto tc_gate = [&](const unsigned char* ts) -> float {
    const uint32_t base = smem_u32(ts);
    const bool need_low = (p.gate != GATE_CS);
    float2 el2 = make_float2(0.f, 0.f), eh2 = make_float2(0.f, 0.f), eh3 = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int np = 0; np < HDL / 16; ++np) {
      float cl[4] = {}, cd[4][4] = {};
#ifdef OC_GATE_ILP
      // low-band partials of the four k-steps in separate accumulators (no
      // dependent MMA chain), added afterwards
      float cls[4][4] = {};
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        uint32_t a[4];
        ldsm_x4_t(base + offG + s4 * 8 * kRowB + ch3[np], a);  // tc_addr(8 s4 + x + 32 b4, 16 np + 8 b3)
        if (need_low) mma16816<KBF16>(cls[s4], a, bLow, bLow);
        mma16816<KBF16>(cd[s4], a, bDiff, bNeg);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) cl[j] = (cls[0][j] + cls[1][j]) + (cls[2][j] + cls[3][j]);
#else
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        uint32_t a[4];
        ldsm_x4_t(base + offG + s4 * 8 * kRowB + ch3[np], a);  // tc_addr(8 s4 + x + 32 b4, 16 np + 8 b3)
        if (need_low) mma16816<KBF16>(cl, a, bLow, bLow);
        mma16816<KBF16>(cd[s4], a, bDiff, bNeg);
      }
#endif
      el2 = __ffma2_rn(make_float2(cl[0], cl[1]), make_float2(cl[0], cl[1]), el2);
      el2 = __ffma2_rn(make_float2(cl[2], cl[3]), make_float2(cl[2], cl[3]), el2);
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        eh2 = __ffma2_rn(make_float2(cd[s4][0], cd[s4][1]), make_float2(cd[s4][0], cd[s4][1]), eh2);
        eh3 = __ffma2_rn(make_float2(cd[s4][2], cd[s4][3]), make_float2(cd[s4][2], cd[s4][3]), eh3);
      }
    }
    const float2 e = warp_sum2(make_float2(el2.x + el2.y, (eh2.x + eh2.y) + (eh3.x + eh3.y)));
    float el = need_low ? e.x : 0.f, eh = e.y;
    if constexpr (P > 1) {  // add the team's panels, in panel order (the same sum in every warp)
      float2* xb = xch + (ktiles & 1) * P;
      if (lane == 0) xb[panel] = make_float2(el, eh);
      team_sync();
      el = 0.f;
      eh = 0.f;
#pragma unroll
      for (int q = 0; q < P; ++q) {
        const float2 v = xb[q];
        el += v.x;
        eh += v.y;
      }
    }
    ++ktiles;
    if (need_low) return __fdiv_rn(eh * 0.5f, el + 1e-6f);
    float kn = sqrtf(eh * 0.5f);
    if (kn < 1e-38f) kn = 0.f;
    return qmax * kn;
  };


  // ======================================================== single pass
  // Team wg owns the flattened K tiles [fa, fb) (unit-major, split-major inside
  // a unit, so a range interleaves over the sequence).  It gates each tile and
  // streams the V of a retained tile into the ring slot its K tile just left;
  // the ring is one FIFO of copies.  A unit's state is written once all its K
  // tiles in the range are gated and no V copy of it is pending: directly when
  // the range holds the whole unit, else as a partial state for merge_kernel.
  int kept_stat = 0;
  if constexpr (ATTN) {
    // units without a tile: zero output (or an empty partial state)
    if (active)
      for (int u = (int)wg; u < U; u += (int)WE) {
        if (tp[u + 1] != tp[u]) continue;
        const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
        for (int g = 0; g < GC && chunk * GC + g < p.group; ++g)
          for (int d = panel * HDL + lane; d < (panel + 1) * HDL; d += 32)
            emit(p, seq, kvh * p.group + chunk * GC + g, d, -1e9f, 0.f, 0.f);
      }
  }
#ifdef OC_TRACE
    tr_x[2] = oc_clock();
#endif
    float m_run[GC], l_part[GC];
    float2 acc[TC ? 1 : GC][D2];
    // tensor-core path: this lane's query g8 (m, partial l) and O^T fragments
    float m_mine = -1e9f, l_mine = 0.f;
    float tacc[TC ? HDL / 16 : 1][4];  // this warp's HDL output columns
    auto reset_state = [&]() {
      if constexpr (TC) {
        m_mine = -1e9f;
        l_mine = 0.f;
#pragma unroll
        for (int mt = 0; mt < HDL / 16; ++mt)
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
    constexpr int PST = HDL + 4;  // floats per (slot, g, panel) partial record: acc[HDL], m, l
    auto rec_of = [&](int64_t sl, int g) { return part + ((sl * GC + g) * P + panel) * PST; };

    // finalize(u, empty): write this warp's state for unit u (empty = no tile of
    // u retained in this warp's range: an empty state, the accumulator untouched)
    auto finalize = [&](int u, bool empty) {
      const int seq = unit_seq(u), kvh = unit_kvh(u), chunk = unit_chunk(u);
      const int gvalid = (p.group - chunk * GC) < GC ? (p.group - chunk * GC) : GC;
      const int hq0 = kvh * p.group + chunk * GC;
      const int64_t R0 = tp[u], R1 = (int64_t)tp[u + 1] - 1;
      const int64_t w0 = range_owner(R0, N, WE), w1 = range_owner(R1, N, WE);
      const bool direct = (w0 == w1);
      const int64_t slot = direct ? 0 : partial_slot(wg, R0, N, WE);
      // put(query, dim, m, l, acc): write the merged state of one output element
      auto put = [&](int qq, int d, float m, float l, float a) {
        if (empty) {
          m = -1e9f;
          l = 0.f;
          a = 0.f;
        }
        if (direct) {
          if (qq < gvalid) emit(p, seq, hq0 + qq, panel * HDL + d, m, l, a);
        } else if (qq < GC) {
          rec_of(slot, qq)[d] = a;
        }
      };
      if constexpr (TC) {
        if (GC <= 4 && !empty) {  // packed P: add the tail columns 4..7 into the head columns 0..3
#pragma unroll
          for (int mt = 0; mt < HDL / 16; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) tacc[mt][j] += __shfl_xor_sync(0xffffffffu, tacc[mt][j], 2);
        }
        float lq = l_mine + __shfl_xor_sync(0xffffffffu, l_mine, 1);
        lq += __shfl_xor_sync(0xffffffffu, lq, 2);
        // one query at a time: the lanes holding its columns stage them in
        // shared memory, then every lane writes two consecutive columns
        static_assert(!TC || HDL == 64 || HDL == 32, "tensor-core panels are 64 or 32 columns");
        const float2* stg2 = reinterpret_cast<const float2*>(stg);
#pragma unroll
        for (int q = 0; q < GC; ++q) {
          if (!empty) {
            if (t4 == (q >> 1)) {
#pragma unroll
              for (int mt = 0; mt < HDL / 16; ++mt) {
                stg[16 * mt + g8] = tacc[mt][q & 1];
                stg[16 * mt + g8 + 8] = tacc[mt][2 + (q & 1)];
              }
            }
            __syncwarp();
          }
          const float2 v = (empty || 2 * lane >= HDL) ? make_float2(0.f, 0.f) : stg2[lane];
          const float mq = __shfl_sync(0xffffffffu, m_mine, 4 * q), lqq = __shfl_sync(0xffffffffu, lq, 4 * q);
          if (2 * lane < HDL) {
            put(q, 2 * lane, mq, lqq, v.x);
            put(q, 2 * lane + 1, mq, lqq, v.y);
          }
          __syncwarp();
        }
        if (!direct && t4 == 0 && g8 < GC)
          *reinterpret_cast<float2*>(rec_of(slot, g8) + HDL) =
              empty ? make_float2(-1e9f, 0.f) : make_float2(m_mine, lq);
      } else {
        // sum the row groups' accumulators and the lanes' probability sums
#pragma unroll
        for (int o = C; o < 32; o <<= 1)
          if (!empty)
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
              *reinterpret_cast<float2*>(rec_of(slot, g) + HDL) =
                  empty ? make_float2(-1e9f, 0.f) : make_float2(m_run[g], lsum[g]);
          }
      }
      // split units are merged by merge_kernel once the grid has completed
    };


  reset_state();


  int u_k = -1, kept_k = 0;  // unit of the last gated K tile and its retained tiles in the range
  int seq_k = 0, kvh_k = 0, chunk_k = 0;
  int f_gated = fa;                  // K tiles [fa, f_gated) are gated
  int acc_unit = -1;                 // unit held by the accumulator
  int uend_k = 0, ua_acc = 0, uend_acc = 0;  // range of the K unit / accumulator unit in [fa, fb)

  for (uint32_t j = 0;; ++j) {
    const uint32_t s = j % NSLOT;
    if (!__any_sync(0xffffffffu, lane < NSLOT && dsc_a >= 0)) break;
    const int da = __shfl_sync(0xffffffffu, dsc_a, s);
    const int db = __shfl_sync(0xffffffffu, dsc_b, s);
    const int f = da < 0 ? -1 : fa + (da >> 1);
    const int isv = da & 1;
    const int u = db >> 20, tile = db & ((1 << 20) - 1);
    if (f < 0) {
      issue_next(s);
      continue;
    }
    unsigned char* ts = wait_slot(s);
#ifdef OC_TRACE
    if (tr_t2 == 0) tr_t2 = oc_clock();
    if (isv) ++tr_nv; else ++tr_nk;
#endif
    const uint32_t ls = (paired && isv) ? (s + NSLOT - 1) % NSLOT : s;  // slot holding this tile's logits
    float* lgs = lgs_base + ls * (CF::LGB / 4);
    if (!isv) {
      // ================================================ K tile: gate (+ logits)
      if (u != u_k) {
        u_k = u;
        uend_k = tp[u + 1] < fb ? tp[u + 1] : fb;
        kept_k = 0;
        seq_k = unit_seq(u);
        kvh_k = unit_kvh(u);
        chunk_k = unit_chunk(u);
      }
      if constexpr (ATTN) {
        if (u != q_unit) {
          q_unit = u;
          const int seq = seq_k, kvh = kvh_k, chunk = chunk_k;
          const int64_t qb = (int64_t)seq * p.q_seq_stride;
          if constexpr (TC) {
            if (u == pf_unit) {  // fragments prefetched when the copy cursor entered the unit
              qf_apply(qf_pf, qok_pf);
            } else {
              bool ok;
              uint32_t tmp[TC ? HDL / 16 : 1][2];
              load_qf(seq, kvh, chunk, tmp, ok);
              qf_apply(tmp, ok);
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
          if (p.gate == GATE_CS && p.group <= 8) {
            // max_g |q_g|: four lanes per query head, one round of independent loads
            const int g = lane >> 2, part = lane & 3;
            float ss = 0.f;
            if (g < p.group) {
              const int64_t row = qb + (int64_t)(kvh * p.group + g) * p.q_head_stride + part * (HD / 4);
#pragma unroll 8
              for (int d = 0; d < HD / 4; ++d) {
                const float x = load_any(p.q, row + d, p.q_dtype);
                ss = fmaf(x, x, ss);
              }
            }
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            ss += __shfl_xor_sync(0xffffffffu, ss, 2);
            float qn = sqrtf(ss);
            if (qn < 1e-38f) qn = 0.f;
            if (g >= p.group) qn = 0.f;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {  // max over the heads; a NaN norm propagates like torch.max
              const float y = __shfl_xor_sync(0xffffffffu, qn, o);
              qn = (qn != qn || y != y) ? __int_as_float(0x7fc00000) : fmaxf(qn, y);
            }
            qmax = qn;
          } else if (p.gate == GATE_CS) {
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

      // ---- band energies
      float score = 0.f;
      if (p.gate != GATE_LIST) {
      if constexpr (TC) {
        OC_TR_BEGIN(tg0);
        score = tc_gate(ts);
        OC_TR_END(0, tg0);
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
        for (int i0 = 0; i0 < PAIRS; i0 += NRES) {
#pragma unroll
          for (int k = 0; k < NRES; ++k) {
            const int i2 = i0 + k;
            float2 a[D2], b[D2];
            Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2) * CF::ROWK + c * 16, a);
            Elem<KT>::template cvt2<DPT>(ts + (rg + RG * i2 + 32) * CF::ROWK + c * 16, b);
            k_dequant<KT>(p, a);
            k_dequant<KT>(p, b);
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
      }
      bool keep;
      if (p.gate == GATE_LIST) keep = true;
      else if (p.gate == GATE_ZETA_ATTN) keep = !(score > p.thr);
      else if (p.gate == GATE_ZETA_MASK) keep = (score <= p.thr);
      else keep = !(score <= p.thr);

      if (lane == 0 && panel == 0 && chunk_k == 0) {
        const int64_t mi = (int64_t)(seq_k * p.num_kv_heads + kvh_k) * p.num_tiles + tile;
        if (p.mask) p.mask[mi] = keep ? 1 : 0;
        if (p.score) p.score[mi] = score;
      }
      f_gated = f + 1;
      bool v_issued = false;
      if (keep) {
        if (chunk_k == 0 && panel == 0) ++kept_stat;
        if constexpr (ATTN) {
          ++kept_k;
          OC_TR_BEGIN(tl0);
          if constexpr (TC) {
            // logits = K (tokens x dims) * q (dims x queries): 4 token tiles of
            // 16, over this warp's panel (the team adds the panels' partials)
            const uint32_t base = smem_u32(ts);
            float cq[4][4] = {};
#pragma unroll
            for (int ks = 0; ks < HDL / 16; ++ks)
#pragma unroll
              for (int mt = 0; mt < 4; ++mt) {
                uint32_t a4[4];
                ldsm_x4(base + offL + mt * 16 * kRowB + ch4[ks], a4);  // tc_addr(16 mt + x + 8 b3, 16 ks + 8 b4)
                mma16816<KBF16>(cq[mt], a4, qf[ks][0], qf[ks][1]);
              }
            // C(token, query): lane holds tokens 16mt+g8 (+8), queries 2t4, 2t4+1
            float* dstl = lgs;
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
              k_dequant<KT>(p, kk);
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
            float* dstl = lgs;
#pragma unroll
            for (int h = 0; h < 2 * GC; h += 2) {
              const int idx = c * 2 * GC + h;
              const int g = idx / RPL, m = idx % RPL;
              *reinterpret_cast<float2*>(dstl + g * 64 + rg * RPL + m) = make_float2(lg[h], lg[h + 1]);
            }
          }
          OC_TR_END(1, tl0);
          if (!paired) {
            OC_TR_BEGIN(ti0);
            __syncwarp();  // K tile read, logits stored: the slot takes this tile's V
            issue(s, seq_k, kvh_k, tile, true);
            OC_TR_END(3, ti0);
            if (lane == (int)s) dsc_a |= 1;
            v_issued = true;
          }
        }
      }
      if (!v_issued) {
        OC_TR_BEGIN(ti1);
        __syncwarp();
        issue_next(s);
        OC_TR_END(3, ti1);
      }
      if constexpr (ATTN) {
        const int uend = uend_k;
        if (f + 1 == uend && kept_k == 0) finalize(u, true);
      }
    } else {
      // ================================================ V tile of a retained tile
      OC_TR_BEGIN(tv0);
      if (acc_unit != u) {
        acc_unit = u;
        ua_acc = tp[u];
        uend_acc = tp[u + 1] < fb ? tp[u + 1] : fb;
      }
      if constexpr (TC) {
        // B = P (tokens x 8 columns).  Up to 4 queries: column n carries the
        // 16-bit head (n < 4) or tail (n >= 4) of query n & 3, so one MMA adds
        // both halves; with more queries head and tail take one MMA each.
        // This lane computes P for query qg = column g8 (mod 4 when packed).
        constexpr bool PACK = GC <= 4;
        const int qg = PACK ? (g8 & 3) : g8;
        const bool qok = qg < GC;
        // logits: the sum of the team's panel partials, in panel order
        team_sync();
        auto lg2 = [&](int o) -> float2 {
          if constexpr (P == 1) {
            return *reinterpret_cast<const float2*>(lgs + o);
          } else {
            float2 t = make_float2(0.f, 0.f);
#pragma unroll
            for (int q = 0; q < P; ++q) {
              const float2 v = *reinterpret_cast<const float2*>(lgs_all + ((team * P + q) * NSLOT + ls) * (CF::LGB / 4) + o);
              t.x += v.x;
              t.y += v.y;
            }
            return t;
          }
        };
        float lv[4][4];
        float lmax = -INFINITY;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const float2 x = qok ? lg2(qg * 64 + 16 * ks + 2 * t4) : make_float2(-INFINITY, -INFINITY);
          const float2 y = qok ? lg2(qg * 64 + 16 * ks + 2 * t4 + 8) : make_float2(-INFINITY, -INFINITY);
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
            pr[j] = qok ? exp2f(lv[ks][j] - nm) : 0.f;
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
          if constexpr (PACK) {
            if (g8 >= 4) {
              bh[ks][0] = bl[ks][0];
              bh[ks][1] = bl[ks][1];
            }
          }
        }
        l_mine = fmaf(l_mine, alpha, psum);
        // rescale the O^T columns 2t4, 2t4+1 by the alphas of their queries
        const float a0 = __shfl_sync(0xffffffffu, alpha, (8 * t4) & 31);
        const float a1 = __shfl_sync(0xffffffffu, alpha, (8 * t4 + 4) & 31);
#pragma unroll
        for (int mt = 0; mt < HDL / 16; ++mt) {
          tacc[mt][0] *= a0; tacc[mt][1] *= a1; tacc[mt][2] *= a0; tacc[mt][3] *= a1;
        }
        // O^T (dims x columns) += V^T (dims x tokens) * P (tokens x columns)
        const uint32_t base = smem_u32(ts);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
          for (int mt = 0; mt < HDL / 16; ++mt) {
            uint32_t a4[4];
            ldsm_x4_t(base + offV + ks * 16 * kRowB + ch3[mt], a4);  // tc_addr(16 ks + x + 8 b4, 16 mt + 8 b3)
            mma16816<KBF16>(tacc[mt], a4, bh[ks][0], bh[ks][1]);
            if constexpr (!PACK) mma16816<KBF16>(tacc[mt], a4, bl[ks][0], bl[ks][1]);
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
      OC_TR_END(2, tv0);
      OC_TR_BEGIN(ti2);
      __syncwarp();
      issue_next(s);
      OC_TR_END(3, ti2);
    }
    OC_TR_BEGIN(tf0);
    if constexpr (ATTN) {
      if (acc_unit >= 0) {
        const int ua = ua_acc, uend = uend_acc;
        if (f_gated >= uend &&
            !__any_sync(0xffffffffu, lane < NSLOT && dsc_a >= 0 && (dsc_a & 1) && fa + (dsc_a >> 1) >= ua &&
                                         fa + (dsc_a >> 1) < uend)) {
          finalize(acc_unit, false);
          acc_unit = -1;
          reset_state();
        }
      }
    }
    OC_TR_END(4, tf0);
  }
  if constexpr (ATTN) {
    // every team of the grid writes its count (no zeroing needed); merge_kernel sums them
    if (p.team_kept != nullptr && panel == 0 && lane == 0) p.team_kept[wg] = kept_stat;
  } else {
    if (p.stats && lane == 0 && kept_stat) atomicAdd(p.stats, (uint32_t)kept_stat);
  }
  // this CTA's decode work is issued: the merge grid may be scheduled (its
  // griddepcontrol.wait still waits for the whole grid to complete)
#ifdef OC_TRACE
  if (p.trace != nullptr && panel == 0 && lane == 0) {
    unsigned long long* r = p.trace + 24 * wg;
    r[0] = tr_t0; r[1] = tr_t1; r[2] = tr_t2; r[3] = oc_clock();
    r[4] = tr_a; r[5] = tr_b; r[6] = tr_nk; r[7] = tr_nv;
    for (int i = 0; i < 4; ++i) r[8 + i] = tr_x[i];
    r[12] = tr_wait; r[13] = tr_sync; r[14] = tr_polls;
    for (int i = 0; i < 6; ++i) r[16 + i] = (unsigned long long)tr_sec[i];
    r[22] = tr_c; r[23] = tr_d;
  }
#endif
  if constexpr (ATTN) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Merge of the units that several teams share, launched as a programmatic
// dependent of decode_kernel: griddepcontrol.wait returns once the decode
// grid has completed and its stores are visible, so the partial states need
// no fences or tickets.  One CTA per (unit, 64-column panel, query head of
// the chunk): its kMergeWarps warps each combine a contiguous share of the
// unit's partial states (log-sum-exp: running max M, weights 2^(m - M)), and
// warp 0 combines the warps' states through shared memory and writes the
// output.  Units held whole by one team were written directly.
constexpr int kMergeWarps = 8;

template <int HD, int GC, int P>
__global__ void __launch_bounds__(32 * kMergeWarps) merge_kernel(const DecodeParams p, int64_t W) {
  constexpr int HDL = HD / P, PST = HDL + 4, MW = kMergeWarps;
#ifdef OC_TRACE
  const unsigned long long tr_m0 = oc_clock();
#endif
  // the next kernel on the stream may be scheduled now; it waits for this grid
  // (griddepcontrol.wait) before it reads what this grid writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
#ifdef OC_TRACE
  if (p.trace != nullptr && threadIdx.x == 0) {
    p.trace[24 * W + 3 * blockIdx.x] = tr_m0;
    p.trace[24 * W + 3 * blockIdx.x + 1] = oc_clock();
  }
#endif
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nchunks = (p.group + GC - 1) / GC;
  const int U = p.num_seqs * p.num_kv_heads * nchunks;
  if (p.stats != nullptr && blockIdx.x == 0 && wid == 0) {  // retained-tile count of the launch
    int s = 0;
    for (int64_t i = lane; i < W; i += 32) s += __ldcg(p.team_kept + i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      if (p.stats_add) *p.stats += (uint32_t)s;
      else *p.stats = (uint32_t)s;
    }
  }
  const int64_t item = blockIdx.x;
  if (item >= (int64_t)U * P * GC) return;
  const int g = (int)(item % GC);
  const int u = (int)(item / (P * GC)), panel = (int)((item / GC) % P);
  const int* tp = p.tile_prefix;
  const int64_t N = tp[U];
  const int64_t WE = (N < W) ? (N > 0 ? N : 1) : W;
  const int64_t R0 = tp[u], R1 = (int64_t)tp[u + 1] - 1;
  if (R1 < R0) return;  // a unit without tiles was written by the decode kernel
  const int64_t w0 = range_owner(R0, N, WE), w1 = range_owner(R1, N, WE);
  if (w0 == w1) return;
  const int seq = u / (p.num_kv_heads * nchunks), kvh = (u / nchunks) % p.num_kv_heads, chunk = u % nchunks;
  const int gvalid = (p.group - chunk * GC) < GC ? (p.group - chunk * GC) : GC;
  if (g >= gvalid) return;
  auto rec_of = [&](int64_t sl) -> const float* { return p.part + ((sl * GC + g) * P + panel) * PST; };
  const int n = (int)(w1 - w0 + 1);
  const int64_t sl0 = partial_slot(w0, R0, N, WE);
  auto slot_i = [&](int i) -> int64_t { return i == 0 ? sl0 : 2 * (w0 + i); };
  constexpr int NE = (HDL + 31) / 32;  // columns per lane
  constexpr int CH = NE <= 2 ? 16 : (NE <= 4 ? 8 : 4);  // partials whose accumulators are loaded together
  const int per = (n + MW - 1) / MW;
  const int i0 = wid * per, i1 = (i0 + per < n) ? i0 + per : n;
  float Mw = -INFINITY, lw = 0.f, a[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) a[e] = 0.f;
  if (i0 < i1) {
    for (int i = i0 + lane; i < i1; i += 32) Mw = fmaxf(Mw, __ldcg(rec_of(slot_i(i)) + HDL));
    Mw = warp_max(Mw);
    for (int b0 = i0; b0 < i1; b0 += CH) {
      float v[CH][NE];
#pragma unroll
      for (int k = 0; k < CH; ++k)
#pragma unroll
        for (int e = 0; e < NE; ++e)
          v[k][e] = (b0 + k < i1 && lane + 32 * e < HDL) ? __ldcg(rec_of(slot_i(b0 + k)) + lane + 32 * e) : 0.f;
      float wt = 0.f;  // lane k < CH: weight of partial b0 + k
      if (lane < CH && b0 + lane < i1) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec_of(slot_i(b0 + lane)) + HDL));
        wt = exp2f(ml.x - Mw);
        lw = fmaf(ml.y, wt, lw);
      }
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const float w = __shfl_sync(0xffffffffu, wt, k);
#pragma unroll
        for (int e = 0; e < NE; ++e) a[e] = fmaf(v[k][e], w, a[e]);
      }
    }
    lw = warp_sum(lw);
  }
  __shared__ float s_m[MW], s_l[MW], s_a[MW][NE * 32];
  if (lane == 0) {
    s_m[wid] = Mw;
    s_l[wid] = lw;
  }
#pragma unroll
  for (int e = 0; e < NE; ++e) s_a[wid][lane + 32 * e] = a[e];
  __syncthreads();
  if (wid != 0) return;
  float M = s_m[0];
#pragma unroll
  for (int w = 1; w < MW; ++w) M = fmaxf(M, s_m[w]);
  float L = 0.f, o[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) o[e] = 0.f;
#pragma unroll
  for (int w = 0; w < MW; ++w) {
    const float f = exp2f(s_m[w] - M);  // a warp without partials has m = -inf: weight 0
    L = fmaf(s_l[w], f, L);
#pragma unroll
    for (int e = 0; e < NE; ++e) o[e] = fmaf(s_a[w][lane + 32 * e], f, o[e]);
  }
#pragma unroll
  for (int e = 0; e < NE; ++e)
    if (lane + 32 * e < HDL) emit(p, seq, kvh * p.group + chunk * GC + g, panel * HDL + lane + 32 * e, M, L, o[e]);
}

template <typename KT, typename VT, int HD, int GC, bool ATTN, int NSLOT, bool TC>
cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int num_sms,
                          cudaStream_t stream) {
  using CF = Cfg<KT, VT, HD, GC, ATTN, NSLOT, TC>;
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
  // about kTilesPerTeam tiles per team, at most one wave of resident CTAs
  constexpr int kTeams = CF::NW / CF::P;
  const int64_t want = (tiles + kTilesPerTeam * kTeams - 1) / (kTilesPerTeam * kTeams);
  // at most one wave of resident CTAs on this device, whatever num_sms says
  static int dev_sms[64] = {0};
  if (dev_sms[dev] == 0) cudaDeviceGetAttribute(&dev_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int sms_cap = (num_sms > 0 && num_sms < dev_sms[dev]) ? num_sms : dev_sms[dev];
  const int64_t cap = (int64_t)sms_cap * resident[dev];
  int64_t grid = want < 1 ? 1 : (want > cap ? cap : want);
  if (grid * (CF::NW / CF::P) > CF::MAXT) grid = CF::MAXT / (CF::NW / CF::P);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(CF::NT);
  cfg.dynamicSmemBytes = CF::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute da[1];
  da[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  da[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = da;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, tk, tv);
  if (e != cudaSuccess || !ATTN) return e;
  // merge of the units shared by several teams: a programmatic dependent launch
  const int64_t items = (int64_t)p.num_seqs * p.num_kv_heads * nchunks * CF::P * GC;
  cudaLaunchConfig_t mc = {};
  mc.gridDim = dim3((unsigned)items);
  mc.blockDim = dim3(32 * kMergeWarps);
  mc.stream = stream;
  cudaLaunchAttribute ma[1];
  ma[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  ma[0].val.programmaticStreamSerializationAllowed = 1;
  mc.attrs = ma;
  mc.numAttrs = 1;
  return cudaLaunchKernelEx(&mc, merge_kernel<HD, GC, CF::P>, p, grid * (int64_t)(CF::NW / CF::P));
}

}  // namespace oc
