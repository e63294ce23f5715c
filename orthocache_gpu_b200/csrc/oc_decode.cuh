// Fused spectral-eviction decode attention for B200 (sm_100a).
//
// One kernel template serves every variant of the reference's hot path
// (j-arndt/orthocache-gpu, src/orthocache_gpu/triton_kernels/):
//   * V1 / V2 zeta-gated split-K decode ........ fused_eviction.py:84-373
//   * V3 Cauchy-Schwarz GQA gate ............... gqa_eviction.py:286-495
//   * paged KV (block-table gather) ............ paged_eviction.py:56-237
//   * mask / zeta scoring only ................. fwht_fused_prototype.py:102-192
//
// Work decomposition: one CTA per (sequence, kv-head, query chunk, split);
// split s processes tiles s, s+S, s+2S, ... of its sequence (the reference's
// interleaved assignment, fused_eviction.py:259).  A CTA streams its K tiles
// HBM -> shared memory with bulk-async copies (the TMA engine,
// cp.async.bulk + mbarrier) through an NS-slot ring, scores each tile, and
// only for retained tiles enqueues the V tile into the same ring.  V of an
// evicted tile is never read.
//
// Band energies use closed forms of the natural-order 64-point Walsh
// transform along the token axis of the tile (no 64x64 matmul):
//   E_high = sum_{s=32..63} sum_d (W K)[s,d]^2 = 1/2 sum_d sum_{t<32} (K[t,d]-K[t+32,d])^2
//            (row s>=32 of H_64 is [h, -h]);
//   E_low  = sum_{r=1..7}  sum_d (W K)[r,d]^2 = 1/64 sum_d sum_{r=1..7} (H_8 S_d)_r^2
//            with S_d[j] = sum_{t = j mod 8} K[t,d] (row r<8 of H_64 is H_8[r, t mod 8]).
// The 8-point transform is an in-register butterfly per head_dim column.
//
// Thread layout (NT = P*C threads): C "chunk lanes" cover one K row (CB bytes
// each, DPT dims), P row groups; thread (c, rg) owns rows rg + P*m, m < R=64/P,
// all with the same residue mod 8, and every pair (t, t+32) it needs for E_high.
//
// Softmax: online, per query head, in the log2 domain (logits pre-scaled by
// log2(e)/sqrt(hd)); m starts at -1e9 and the result is acc / max(l, 1e-9)
// exactly as fused_eviction.py:242-309,369-370.  Split partials (m, l, acc)
// are merged by the last CTA of each (sequence, kv-head, chunk) to arrive
// (atomic ticket), so one launch produces the final output.
//
// Every wait is bounded: a wait that runs out sets a status bit, drains the
// CTA's own copies (again bounded) and returns.  No spin on another CTA.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

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
  float* part_ml;     // (units, num_splits, 2)   units = seqs*kv_heads*group
  float* part_acc;    // (units, num_splits, head_dim)
  uint32_t* tickets;  // (seqs*kv_heads*chunks), zero between launches
  // shard mode (nullable): write the merged partial state (m, l, unnormalised
  // acc) of each query head instead of the normalised output
  float* sh_m;
  float* sh_l;
  float* sh_acc;
};

// ---------------------------------------------------------------- conversions
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int B = 4;
  template <int N> __device__ static void cvt(const unsigned char* s, float* f) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      float4 x = *reinterpret_cast<const float4*>(s + 4 * i);
      f[i] = x.x; f[i + 1] = x.y; f[i + 2] = x.z; f[i + 3] = x.w;
    }
  }
};
template <> struct Elem<__half> {
  static constexpr int B = 2;
  template <int N> __device__ static void cvt(const unsigned char* s, float* f) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      uint4 x = *reinterpret_cast<const uint4*>(s + 2 * i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        f[i + 2 * j] = t.x; f[i + 2 * j + 1] = t.y;
      }
    }
  }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int B = 2;
  template <int N> __device__ static void cvt(const unsigned char* s, float* f) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      uint4 x = *reinterpret_cast<const uint4*>(s + 2 * i);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[i + 2 * j] = __uint_as_float(w[j] << 16);
        f[i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
    }
  }
};
template <> struct Elem<__nv_fp8_e4m3> {
  static constexpr int B = 1;
  template <int N> __device__ static void cvt(const unsigned char* s, float* f) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      uint2 x = *reinterpret_cast<const uint2*>(s + i);
      const uint32_t w[2] = {x.x, x.y};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
              static_cast<__nv_fp8x2_storage_t>((w[j] >> (16 * h)) & 0xffffu), __NV_E4M3);
          float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hr));
          f[i + 4 * j + 2 * h] = t.x; f[i + 4 * j + 2 * h + 1] = t.y;
        }
      }
    }
  }
};

// CB packed bytes of one K row chunk, held in registers.
template <int CB> struct Raw;
template <> struct Raw<16> {
  uint4 v;
  __device__ static Raw load(const unsigned char* s) { return Raw{*reinterpret_cast<const uint4*>(s)}; }
  __device__ const unsigned char* bytes() const { return reinterpret_cast<const unsigned char*>(&v); }
};
template <> struct Raw<8> {
  uint2 v;
  __device__ static Raw load(const unsigned char* s) { return Raw{*reinterpret_cast<const uint2*>(s)}; }
  __device__ const unsigned char* bytes() const { return reinterpret_cast<const unsigned char*>(&v); }
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

// ---------------------------------------------------------------- config
template <typename KT, typename VT, int HD, int GC, bool ATTN>
struct Cfg {
  static constexpr int KB = Elem<KT>::B;
  static constexpr int VB = Elem<VT>::B;
  static constexpr int CB = (KB == 1) ? 8 : 16;  // bytes of a K row per chunk lane
  static constexpr int DPT = CB / KB;            // head_dim columns per thread
  static constexpr int ROWK = HD * KB;
  static constexpr int ROWV = HD * VB;
  static constexpr int C = ROWK / CB;
  static constexpr int P = (C >= 4) ? 8 : 32 / C;
  static constexpr int NT = P * C;
  static constexpr int R = 64 / P;
  static constexpr int NW = NT / 32;
  static constexpr int VCB = DPT * VB;
  static constexpr int ROWMAX = (ATTN && ROWV > ROWK) ? ROWV : ROWK;
  static constexpr int SLOT = 64 * ROWMAX;
  static constexpr int NS = SLOT >= 65536 ? 2 : (65536 / SLOT < 3 ? 3 : (65536 / SLOT > 8 ? 8 : 65536 / SLOT));
  static constexpr int NLG = NS + 2;
  // shared memory carve-up (bytes)
  static constexpr int OFF_BAR = NS * SLOT;
  static constexpr int OFF_S = OFF_BAR + 8 * NS;                    // P*HD floats
  static constexpr int OFF_LG = OFF_S + 4 * P * HD;                 // NLG*GC*64 floats
  static constexpr int OFF_MX = OFF_LG + (ATTN ? 4 * NLG * GC * 64 : 0);  // NLG*NW*GC
  static constexpr int OFF_EH = OFF_MX + (ATTN ? 4 * NLG * NW * GC : 0);  // 2*NW
  static constexpr int OFF_EL = OFF_EH + 4 * 2 * NW;                // 2*NW
  static constexpr int OFF_KT = OFF_EL + 4 * 2 * NW;                // NLG ints
  static constexpr int OFF_MISC = OFF_KT + 4 * NLG;                 // 8 words
  static constexpr int SMEM = OFF_MISC + 32;
  static_assert(C >= 1 && C <= 32 && (C & (C - 1)) == 0, "row bytes per chunk layout");
  static_assert(NT >= 32 && NT <= 1024, "threads");
  static_assert(NT >= HD, "one thread per head_dim column in the merge");
  static_assert(!ATTN || 4 * (P * GC * HD + P * GC) <= NS * SLOT, "final reduction fits in the ring");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// ---------------------------------------------------------------- kernel
template <typename KT, typename VT, int HD, int GC, bool ATTN>
__global__ void __launch_bounds__(Cfg<KT, VT, HD, GC, ATTN>::NT, 1)
    decode_kernel(const DecodeParams p) {
  using CF = Cfg<KT, VT, HD, GC, ATTN>;
  constexpr int C = CF::C, P = CF::P, R = CF::R, DPT = CF::DPT, NT = CF::NT, NW = CF::NW;
  constexpr int NS = CF::NS, NLG = CF::NLG, SLOT = CF::SLOT;
  extern __shared__ __align__(128) unsigned char smem[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid % C, rg = tid / C;

  const int nchunks = (p.group + GC - 1) / GC;
  int bx = blockIdx.x;
  const int chunk = bx % nchunks;
  bx /= nchunks;
  const int kvh = bx % p.num_kv_heads;
  const int seq = bx / p.num_kv_heads;
  const int split = blockIdx.y;
  const int S = p.num_splits;
  const int grp = (seq * p.num_kv_heads + kvh);  // (seq, kv-head) index

  int T = p.num_tiles;
  if (p.seq_lens != nullptr) {
    const int L = p.seq_lens[seq];
    if (L < 0 || (L & 63) || L > p.num_tiles * 64) {
      if (tid == 0 && split == 0 && chunk == 0) atomicOr(p.status, ST_BAD_SEQLEN);
    }
    const int lt = L < 0 ? 0 : (L >> 6);
    T = lt < T ? lt : T;
  }
  const int my_tiles = split < T ? (T - split + S - 1) / S : 0;

  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + CF::OFF_BAR;
  float* sS = reinterpret_cast<float*>(smem + CF::OFF_S);
  float* sLG = reinterpret_cast<float*>(smem + CF::OFF_LG);
  float* sMX = reinterpret_cast<float*>(smem + CF::OFF_MX);
  float* sEH = reinterpret_cast<float*>(smem + CF::OFF_EH);
  float* sEL = reinterpret_cast<float*>(smem + CF::OFF_EL);
  int* sKT = reinterpret_cast<int*>(smem + CF::OFF_KT);
  uint32_t* sMisc = reinterpret_cast<uint32_t*>(smem + CF::OFF_MISC);

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(bars + 8 * s, 1);
    mbar_init_fence();
  }

  // ---- queries of this chunk: my DPT columns, pre-scaled for exp2
  float qv[GC][DPT];
  float qmax = 0.f;  // max_g |q_g| over the whole group (Cauchy-Schwarz gate)
  if constexpr (ATTN) {
    const int64_t qbase = (int64_t)seq * p.q_seq_stride;
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      const int hq = chunk * GC + g;
#pragma unroll
      for (int d = 0; d < DPT; ++d)
        qv[g][d] = (hq < p.group)
                       ? load_any(p.q, qbase + (int64_t)(kvh * p.group + hq) * p.q_head_stride + c * DPT + d,
                                  p.q_dtype) * p.scale_log2
                       : 0.f;
    }
    if (p.gate == GATE_CS) {
      for (int g = 0; g < p.group; ++g) {
        float ss = 0.f;
#pragma unroll
        for (int d = 0; d < DPT; ++d) {
          const float x = load_any(p.q, qbase + (int64_t)(kvh * p.group + g) * p.q_head_stride + c * DPT + d,
                                   p.q_dtype);
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
  __syncthreads();

  const uint64_t pol = policy_evict_first();

  // ---- issue machinery (executed uniformly by all threads; warp 0 copies)
  uint32_t n_iss = 0, n_done = 0, n_freed = 0, isv_mask = 0;
  int k_iss = 0, v_iss = 0, kept = 0;
  const int64_t kv_seq_k = (int64_t)seq * p.k_seq_stride + (int64_t)kvh * p.k_head_stride;
  const int64_t kv_seq_v = (int64_t)seq * p.v_seq_stride + (int64_t)kvh * p.v_head_stride;

  auto issue = [&](uint32_t slot, int tile, bool isv) {
    if (warp != 0) return;
    const uint32_t bar = bars + 8 * slot, dst = ring + slot * SLOT;
    const int row = isv ? CF::ROWV : CF::ROWK;
    if (lane == 0) mbar_arrive_expect_tx(bar, 64u * row);
    __syncwarp();
    const char* basep = isv ? p.v : p.k;
    const int64_t tok = isv ? p.v_tok_stride : p.k_tok_stride;
    if (p.layout == LAYOUT_LINEAR) {
      const char* base = basep + (isv ? kv_seq_v : kv_seq_k);
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
  };

  auto refill = [&]() {
    while (n_iss - n_freed < (uint32_t)NS) {
      bool isv;
      int tile;
      if (ATTN && v_iss < kept) {
        isv = true;
        tile = sKT[v_iss % NLG];
        ++v_iss;
      } else if (k_iss < my_tiles) {
        isv = false;
        tile = split + k_iss * S;
        ++k_iss;
      } else {
        break;
      }
      const uint32_t bit = 1u << (n_iss & 31);
      isv_mask = isv ? (isv_mask | bit) : (isv_mask & ~bit);
      issue(n_iss % NS, tile, isv);
      ++n_iss;
    }
  };

  // ---- per-query online softmax state (log2 domain)
  float m_run[GC], l_run[GC], acc[GC][DPT];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m_run[g] = -1e9f;
    l_run[g] = 0.f;
#pragma unroll
    for (int d = 0; d < DPT; ++d) acc[g][d] = 0.f;
  }

  int k_done = 0, v_done = 0, n_kept_total = 0;
  bool bad = false, to_pending = false;
  refill();

  while (k_done < my_tiles || (ATTN && v_done < kept)) {
    const uint32_t slot = n_done % NS;
    const uint32_t parity = (n_done / NS) & 1u;
    const bool is_v = ATTN && ((isv_mask >> (n_done & 31)) & 1u);
    const unsigned char* tile_s = smem + slot * SLOT;

    if (!is_v) {
      // ================= gate a K tile
      const int tile = split + k_done * S;
      const int par = k_done & 1;
      bool to = to_pending || !mbar_wait_bounded(bars + 8 * slot, parity, kWaitLimit);
      float s[DPT];
      float eh = 0.f;
#pragma unroll
      for (int d = 0; d < DPT; ++d) s[d] = 0.f;
      // my K rows stay packed in registers and are converted on use
      Raw<CF::CB> kraw[R];
#pragma unroll
      for (int m = 0; m < R; ++m) kraw[m] = Raw<CF::CB>::load(tile_s + (rg + P * m) * CF::ROWK + c * CF::CB);
      const bool zgate = (p.gate != GATE_CS);
#pragma unroll
      for (int m = 0; m < R / 2; ++m) {
        float a[DPT], b[DPT];
        Elem<KT>::template cvt<DPT>(kraw[m].bytes(), a);
        Elem<KT>::template cvt<DPT>(kraw[m + R / 2].bytes(), b);
#pragma unroll
        for (int d = 0; d < DPT; ++d) {
          const float df = a[d] - b[d];
          eh = fmaf(df, df, eh);
          s[d] += a[d] + b[d];
        }
      }
      if (zgate) {
#pragma unroll
        for (int d = 0; d < DPT; ++d) sS[rg * HD + c * DPT + d] = s[d];
      }
      eh = warp_sum(eh);
      if (lane == 0) sEH[par * NW + warp] = eh;
      // B1: K slot consumed by every thread
      to = __syncthreads_or(to);
      if (to) { bad = true; break; }
      n_freed = n_done + 1;
      refill();

      float score;
      if (zgate) {
        float el = 0.f;
        for (int d = tid; d < HD; d += NT) {
          float u[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) u[j] = 0.f;
#pragma unroll
          for (int r = 0; r < P; ++r) u[r & 7] += sS[r * HD + d];
#pragma unroll
          for (int h = 1; h < 8; h <<= 1)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (!(i & h)) {
                const float a = u[i], b = u[i + h];
                u[i] = a + b;
                u[i + h] = a - b;
              }
#pragma unroll
          for (int r = 1; r < 8; ++r) el = fmaf(u[r], u[r], el);
        }
        el = warp_sum(el);
        if (lane == 0) sEL[par * NW + warp] = el;
        __syncthreads();  // B2
        float elt = 0.f, eht = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          elt += sEL[par * NW + w];
          eht += sEH[par * NW + w];
        }
        const float e_low = elt * (1.f / 64.f);
        const float e_high = eht * 0.5f;
        score = __fdiv_rn(e_high, e_low + 1e-6f);
      } else {
        float eht = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) eht += sEH[par * NW + w];
        float kn = sqrtf(eht * 0.5f);
        if (kn < 1e-38f) kn = 0.f;
        score = qmax * kn;
      }
      bool keep;
      if (p.gate == GATE_ZETA_ATTN) keep = !(score > p.thr);
      else if (p.gate == GATE_ZETA_MASK) keep = (score <= p.thr);
      else keep = !(score <= p.thr);

      if (tid == 0 && chunk == 0) {
        const int64_t mi = (int64_t)grp * p.num_tiles + tile;
        if (p.mask) p.mask[mi] = keep ? 1 : 0;
        if (p.score) p.score[mi] = score;
      }
      n_kept_total += keep ? 1 : 0;

      if constexpr (ATTN) {
        if (keep) {
          const int ks = kept % NLG;
          if (tid == 0) sKT[ks] = tile;
          // logits of my rows / columns, then reduce-scatter over the C chunk lanes
          constexpr int NVAL = GC * R;
          float lg[NVAL];
#pragma unroll
          for (int m = 0; m < R; ++m) {
            float kf[DPT];
            Elem<KT>::template cvt<DPT>(kraw[m].bytes(), kf);
#pragma unroll
            for (int g = 0; g < GC; ++g) {
              float a = 0.f;
#pragma unroll
              for (int d = 0; d < DPT; ++d) a = fmaf(qv[g][d], kf[d], a);
              lg[g * R + m] = a;
            }
          }
          reduce_scatter<NVAL, C>(lg, c);
          constexpr int HELD = NVAL >= C ? NVAL / C : 1;
          const int idx0 = NVAL >= C ? c * (NVAL / C) : c / (C / NVAL);
          const bool writer = NVAL >= C ? true : (c % (C / NVAL) == 0);
          float* lgs = sLG + ks * GC * 64;
          float mx[GC];
#pragma unroll
          for (int g = 0; g < GC; ++g) mx[g] = -INFINITY;
#pragma unroll
          for (int i = 0; i < HELD; ++i) {
            const int idx = idx0 + i;
            const int g = idx / R, m = idx % R;
            if (writer) lgs[g * 64 + rg + P * m] = lg[i];
#pragma unroll
            for (int gg = 0; gg < GC; ++gg)
              if (gg == g) mx[gg] = fmaxf(mx[gg], lg[i]);
          }
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const float w = warp_max(mx[g]);
            if (lane == 0) sMX[(ks * NW + warp) * GC + g] = w;
          }
          ++kept;
          __syncwarp();
          refill();
        }
      }
      ++k_done;
      ++n_done;
    } else {
      if constexpr (ATTN) {
        // ================= PV of a retained tile
        // B0: the gate's logits are visible and the previous slot is consumed
        if (__syncthreads_or(to_pending)) { bad = true; break; }
        n_freed = n_done;
        refill();
        // a wait that runs out is reported at the next barrier
        to_pending = !mbar_wait_bounded(bars + 8 * slot, parity, kWaitLimit);
        const int ks = v_done % NLG;
        const float* lgs = sLG + ks * GC * 64;
        float pr[GC][R];
        float alpha[GC];
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          float tmax = -INFINITY;
#pragma unroll
          for (int w = 0; w < NW; ++w) tmax = fmaxf(tmax, sMX[(ks * NW + w) * GC + g]);
          const float nm = fmaxf(m_run[g], tmax);
          alpha[g] = exp2f(m_run[g] - nm);
          float ps = 0.f;
#pragma unroll
          for (int m = 0; m < R; ++m) {
            pr[g][m] = exp2f(lgs[g * 64 + rg + P * m] - nm);
            ps += pr[g][m];
          }
          l_run[g] = fmaf(l_run[g], alpha[g], ps);
          m_run[g] = nm;
#pragma unroll
          for (int d = 0; d < DPT; ++d) acc[g][d] *= alpha[g];
        }
#pragma unroll
        for (int m = 0; m < R; ++m) {
          float vf[DPT];
          Elem<VT>::template cvt<DPT>(tile_s + (rg + P * m) * CF::ROWV + c * CF::VCB, vf);
#pragma unroll
          for (int g = 0; g < GC; ++g)
#pragma unroll
            for (int d = 0; d < DPT; ++d) acc[g][d] = fmaf(pr[g][m], vf[d], acc[g][d]);
        }
        ++v_done;
        ++n_done;
      }
    }
  }

  if (bad || __syncthreads_or(to_pending)) {
    // bounded drain of this CTA's copies still in flight, then leave
    if (tid == 0) atomicOr(p.status, ST_TIMEOUT);
    for (uint32_t n = n_done; n < n_iss; ++n) mbar_wait_bounded(bars + 8 * (n % NS), (n / NS) & 1u, kWaitLimit);
    return;
  }

  if (p.stats && tid == 0 && chunk == 0 && n_kept_total) atomicAdd(p.stats, (uint32_t)n_kept_total);
  if constexpr (!ATTN) return;

  if constexpr (ATTN) {
    // ---- reduce the P row groups (ring is idle now)
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);  // [P][GC][HD]
    float* redl = red + P * GC * HD;              // [P][GC]
#pragma unroll
    for (int g = 0; g < GC; ++g) {
#pragma unroll
      for (int d = 0; d < DPT; ++d) red[(rg * GC + g) * HD + c * DPT + d] = acc[g][d];
      if (c == 0) redl[rg * GC + g] = l_run[g];
    }
    __syncthreads();
    const int gvalid = (p.group - chunk * GC) < GC ? (p.group - chunk * GC) : GC;
    for (int idx = tid; idx < GC * HD; idx += NT) {
      const int g = idx / HD, d = idx % HD;
      if (g >= gvalid) continue;
      float a = 0.f, l = 0.f;
#pragma unroll
      for (int r = 0; r < P; ++r) {
        a += red[(r * GC + g) * HD + d];
        l += redl[r * GC + g];
      }
      const int hq = kvh * p.group + chunk * GC + g;
      if (S == 1) {
        emit(p, seq, hq, d, m_run[g], l, a);
      } else {
        const int64_t unit = (int64_t)(seq * p.num_kv_heads) * p.group + hq;
        p.part_acc[(unit * S + split) * HD + d] = a;
        if (d == 0) {
          p.part_ml[(unit * S + split) * 2] = m_run[g];
          p.part_ml[(unit * S + split) * 2 + 1] = l;
        }
      }
    }
    if (S == 1) return;

    // ---- last CTA of this (seq, kv-head, chunk) merges the S partials
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const uint32_t prev = atomicAdd(&p.tickets[(int64_t)grp * nchunks + chunk], 1u);
      sMisc[0] = (prev == (uint32_t)(S - 1)) ? 1u : 0u;
    }
    __syncthreads();
    if (sMisc[0] == 0) return;
    __threadfence();
    if (tid == 0) p.tickets[(int64_t)grp * nchunks + chunk] = 0u;

    // HD/4 column lanes x NG split groups, float4 loads
    constexpr int NC4 = HD / 4 > 0 ? HD / 4 : 1;
    constexpr int NG = NT / NC4 > 0 ? NT / NC4 : 1;
    float* mrg = reinterpret_cast<float*>(smem);  // [NG][HD] + [NG] + [NW]
    float* mrgl = mrg + NG * HD;
    float* smax = mrgl + NG;
    for (int g = 0; g < gvalid; ++g) {
      const int hq = kvh * p.group + chunk * GC + g;
      const int64_t unit = (int64_t)(seq * p.num_kv_heads) * p.group + hq;
      const float* ml = p.part_ml + unit * S * 2;
      const float* pa = p.part_acc + unit * S * HD;
      float mloc = -INFINITY;
      for (int s2 = tid; s2 < S; s2 += NT) mloc = fmaxf(mloc, __ldcg(ml + 2 * s2));
      mloc = warp_max(mloc);
      if (lane == 0) smax[warp] = mloc;
      __syncthreads();
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, smax[w]);
      const int c4 = tid % NC4, sg = tid / NC4;
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float lsum = 0.f;
      if (sg < NG && 4 * c4 < HD) {
#pragma unroll 4
        for (int s2 = sg; s2 < S; s2 += NG) {
          const float2 mlv = __ldcg(reinterpret_cast<const float2*>(ml + 2 * s2));
          const float w = exp2f(mlv.x - M);
          const float4 x = __ldcg(reinterpret_cast<const float4*>(pa + (int64_t)s2 * HD + 4 * c4));
          a4.x = fmaf(x.x, w, a4.x); a4.y = fmaf(x.y, w, a4.y);
          a4.z = fmaf(x.z, w, a4.z); a4.w = fmaf(x.w, w, a4.w);
          lsum = fmaf(mlv.y, w, lsum);
        }
        reinterpret_cast<float4*>(mrg + sg * HD)[c4] = a4;
        if (c4 == 0) mrgl[sg] = lsum;
      }
      __syncthreads();
      for (int d = tid; d < HD; d += NT) {
        float a = 0.f, l = 0.f;
        for (int q2 = 0; q2 < NG; ++q2) {
          a += mrg[q2 * HD + d];
          l += mrgl[q2];
        }
        emit(p, seq, hq, d, M, l, a);
      }
      __syncthreads();
    }
  }
}

template <typename KT, typename VT, int HD, int GC, bool ATTN>
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream) {
  using CF = Cfg<KT, VT, HD, GC, ATTN>;
  auto kern = decode_kernel<KT, VT, HD, GC, ATTN>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int nchunks = (p.group + GC - 1) / GC;
  dim3 grid((unsigned)(p.num_seqs * p.num_kv_heads * nchunks), (unsigned)p.num_splits);
  kern<<<grid, CF::NT, CF::SMEM, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace oc
