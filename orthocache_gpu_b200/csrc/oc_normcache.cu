// Spectral norm cache and the O(1) decode gate.
//
//   * tile_high_norm_kernel: per 64-token key tile, |(W K)[hs:he]|_F with W the
//     natural-order 64-point Walsh matrix (1/8 scaled) along the token axis:
//     the prefill-side scoring that fills the norm cache
//     (norm_cache.py:58-117 update_prefill / populate_from_keys; the same
//     transform as fwht_fused_prototype.py:199-248).
//   * decode_gate_kernel: the decode-time gate from cached norms
//     (decode_gate.py:54-106 compute_q_high_norm_exact, :251-300
//     _pytorch_decode_gate): per kv head the statistic s = max (or median)
//     over its G query heads of |q_high|_2 (tight, block-sum projection) or
//     |q|_2, then evict[t] = float32(s * norm[t]) <= float32(tau * 64 * hd).
//     It also compacts the retained tiles of each kv head into a list, in
//     tile order, so that the decode kernel (GATE_LIST) reads K and V of the
//     retained tiles only.
#include <cmath>
#include <cstdint>

#include "../../include/orthocache_b200.h"
#include "oc_decode.cuh"
#include "oc_dispatch.h"

namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(*p);
  else return __half2float(__half(__nv_cvt_fp8_to_halfraw(*reinterpret_cast<const __nv_fp8_storage_t*>(p), __NV_E4M3)));
}

// One CTA per (head, tile): the tile is staged in shared memory as float32,
// every thread transforms one column (64-point Walsh-Hadamard butterflies in
// registers, natural order), squares the rows of the band and the CTA adds
// the columns.  Threads: max(32, head_dim) rounded to whole warps.
template <typename KT>
__global__ void __launch_bounds__(256) tile_high_norm_kernel(const KT* __restrict__ k, int64_t head_stride,
                                                            int64_t tok_stride, int hd, int tiles,
                                                            int hs, int he, float* __restrict__ out,
                                                            int64_t out_stride) {
  extern __shared__ float tile[];  // [64][hd]
  __shared__ float red[8];
  const int h = blockIdx.y, t = blockIdx.x;
  const KT* base = k + (int64_t)h * head_stride + (int64_t)t * 64 * tok_stride;
  for (int i = threadIdx.x; i < 64 * hd; i += blockDim.x) {
    const int r = i / hd, c = i - r * hd;
    tile[i] = ld(base + (int64_t)r * tok_stride + c);
  }
  __syncthreads();
  float e = 0.f;
  const int c = threadIdx.x;
  if (c < hd) {
    float v[64];
#pragma unroll
    for (int r = 0; r < 64; ++r) v[r] = tile[r * hd + c];
#pragma unroll
    for (int s = 1; s < 64; s <<= 1)
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (!(i & s)) {
          const float a = v[i], b = v[i + s];
          v[i] = a + b;
          v[i + s] = a - b;
        }
#pragma unroll
    for (int r = 0; r < 64; ++r)
      if (r >= hs && r < he) e = fmaf(v[r], v[r], e);
  }
  e *= (1.f / 64.f);  // W = H / 8
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = e;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    float n = sqrtf(s);
    if (n < 1e-38f) n = 0.f;  // the reference's subnormal clamp (norm_cache.py:83-85)
    out[(int64_t)h * out_stride + t] = n;
  }
}

// Norm of one query head: tight (|q|^2 - sum_i S_i^2 / bs, S_i the sums of
// low_band contiguous blocks of bs = hd / low_band dims, clamped at 0) or
// loose (|q|^2).  Returns the square root.  One warp.
__device__ float q_norm_warp(const void* q, int dt, int64_t off, int hd, bool tight, int low_band) {
  const int lane = threadIdx.x & 31;
  const int bs = hd / low_band;
  float sq = 0.f, bsum[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) bsum[i] = 0.f;
  for (int d = lane; d < hd; d += 32) {
    const float x = oc::load_any(q, off + d, dt);
    sq = fmaf(x, x, sq);
    const int b = d / bs;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i == b) bsum[i] += x;
  }
  sq = oc::warp_sum(sq);
  if (!tight) return sqrtf(sq);
  float low = 0.f;
  for (int i = 0; i < low_band && i < 32; ++i) {
    const float s = oc::warp_sum(bsum[i]);
    low = fmaf(s, s, low);
  }
  low = low / (float)bs;
  const float hi = fmaxf(sq - low, 0.f);
  return sqrtf(hi);
}

// One CTA per (sequence, kv head).  Writes q_norms[g], evict[t] for t <
// max_tiles (0 beyond num_tiles), and, when list != null, the retained tiles
// in increasing order plus their count.
__global__ void __launch_bounds__(256) decode_gate_kernel(
    const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride, int num_kv_heads, int group,
    int hd, const float* __restrict__ norms, int64_t norm_seq_stride, int64_t norm_head_stride, int num_tiles,
    int max_tiles, float thr, int tight, int low_band, int stat_median, uint8_t* evict,
    int64_t evict_stride, float* q_norms, int* list, int64_t list_stride, int* count) {
  __shared__ float qn[64];
  __shared__ float s_stat;
  __shared__ int wsum[8];
  // the decode grid that consumes the lists may start its prologue now; its
  // griddepcontrol.wait still waits for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int seq = blockIdx.x / num_kv_heads, kvh = blockIdx.x % num_kv_heads;
  const int g_idx = blockIdx.x;  // (seq, kv head) row of the outputs
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int g = warp; g < group; g += nw) {
    const int64_t off = (int64_t)seq * q_seq_stride + (int64_t)(kvh * group + g) * q_head_stride;
    const float n = q_norm_warp(q, q_dtype, off, hd, tight != 0, low_band);
    if (lane == 0) qn[g] = n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s;
    if (!stat_median) {  // torch.max: a NaN propagates
      s = qn[0];
      for (int g = 1; g < group; ++g) s = (s != s || qn[g] != qn[g]) ? __int_as_float(0x7fc00000) : fmaxf(s, qn[g]);
    } else {  // sorted(...)[G // 2]
      const int want = group / 2;
      s = qn[0];
      for (int g = 0; g < group; ++g) {  // the element with exactly `want` smaller (ties by index)
        int below = 0;
        for (int j = 0; j < group; ++j) below += (qn[j] < qn[g]) || (qn[j] == qn[g] && j < g);
        if (below == want) s = qn[g];
      }
    }
    s_stat = s;
    if (q_norms) q_norms[g_idx] = s;
  }
  __syncthreads();
  const float s = s_stat;
  const float* nr = norms + (int64_t)seq * norm_seq_stride + (int64_t)kvh * norm_head_stride;
  int base = 0;
  for (int t0 = 0; t0 < max_tiles; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    bool ev = false, keep = false;
    if (t < num_tiles) {
      const float b = s * nr[t];
      ev = b <= thr;
      keep = !ev;
    }
    if (evict && t < max_tiles) evict[(int64_t)g_idx * evict_stride + t] = ev ? 1 : 0;
    if (list) {
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (lane == 0) wsum[warp] = __popc(m);
      __syncthreads();
      int off = base;
      for (int w = 0; w < warp; ++w) off += wsum[w];
      if (keep) list[(int64_t)g_idx * list_stride + off + __popc(m & ((1u << lane) - 1u))] = t;
      int tot = 0;
      for (int w = 0; w < nw; ++w) tot += wsum[w];
      base += tot;
      __syncthreads();
    }
  }
  if (list && threadIdx.x == 0) count[g_idx] = base;
}

}  // namespace

namespace oc {

int launch_tile_high_norms(const void* keys, int k_dtype, int num_heads, int tiles, int hd, int64_t head_stride,
                           int64_t tok_stride, int hs, int he, float* out, int64_t out_stride, cudaStream_t st) {
  if (tiles == 0 || num_heads == 0) return OC_OK;
  if (num_heads > 65535) return OC_ERR_INVALID;
  const int threads = ((hd < 32 ? 32 : hd) + 31) / 32 * 32;
  const size_t smem = (size_t)64 * hd * sizeof(float);
  const dim3 grid((unsigned)tiles, (unsigned)num_heads);
  cudaError_t e = cudaSuccess;
#define OC_NORM(T)                                                                                         \
  {                                                                                                        \
    auto kern = tile_high_norm_kernel<T>;                                                                  \
    if (smem > 48 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e == cudaSuccess) {                                                                                \
      kern<<<grid, threads, smem, st>>>(static_cast<const T*>(keys), head_stride, tok_stride, hd, tiles, hs, he, \
                                        out, out_stride);                                                  \
      e = cudaGetLastError();                                                                              \
    }                                                                                                      \
  }
  switch (k_dtype) {
    case OC_F32: OC_NORM(float) break;
    case OC_F16: OC_NORM(__half) break;
    case OC_BF16: OC_NORM(__nv_bfloat16) break;
    case OC_F8E4M3: OC_NORM(__nv_fp8_e4m3) break;
    default: return OC_ERR_UNSUPPORTED;
  }
#undef OC_NORM
  return e == cudaSuccess ? OC_OK : OC_ERR_CUDA;
}

int launch_decode_gate(const GateArgs& a, cudaStream_t st) {
  if (a.num_seqs * a.num_kv_heads == 0) return OC_OK;
  decode_gate_kernel<<<(unsigned)(a.num_seqs * a.num_kv_heads), 256, 0, st>>>(
      a.q, a.q_dtype, a.q_seq_stride, a.q_head_stride, a.num_kv_heads, a.group, a.head_dim, a.norms,
      a.norm_seq_stride, a.norm_head_stride, a.num_tiles, a.max_tiles, a.thr, a.tight, a.low_band, a.stat_median,
      a.evict, a.evict_stride, a.q_norms, a.list, a.list_stride, a.count);
  return cudaGetLastError() == cudaSuccess ? OC_OK : OC_ERR_CUDA;
}

}  // namespace oc
