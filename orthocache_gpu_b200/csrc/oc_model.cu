// Decoder-step kernels of the Llama-shaped model driver (model.py): the
// small per-layer operations around the fused decode attention, each one
// launch instead of a chain of PyTorch elementwise ops.
//   oc_add_rms_norm       x += y (optional), h = rmsnorm(x) * weight
//   oc_rope_cache_append  rotary embedding of the step's q / k, k and v
//                         written into the token-major caches at the step's
//                         position (read on the device: CUDA-graph friendly)
//   oc_tail_merge         attention over the ragged tail (the < 64 tokens
//                         after the last whole tile), merged by log-sum-exp
//                         with the fused kernel's softmax state
// They follow the PyTorch ops of the reference harness's Llama decode
// (eval/perplexity_eval.py: RMSNorm, rotate-half rotary embedding) in fp32
// arithmetic with the same rounding points to 16-bit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>

#include "../../include/orthocache_b200.h"

namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <>
__device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) {
  return __half2float(p[i]);
}
template <typename T>
__device__ __forceinline__ T rnd(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 rnd<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half rnd<__half>(float x) {
  return __float2half_rn(x);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

// One CTA per row.  x (rows, n) is updated in place when y is given.
template <typename T>
__global__ void add_rms_norm_kernel(T* x, const T* y, const T* w, T* h, int64_t n, float eps) {
  __shared__ float red[32];
  T* xr = x + blockIdx.x * n;
  const T* yr = y ? y + blockIdx.x * n : nullptr;
  T* hr = h + blockIdx.x * n;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float v = ld(xr, i);
    if (yr) {
      v = ld(xr, i) + ld(yr, i);  // the residual add rounds to the model dtype
      const T r = rnd<T>(v);
      xr[i] = r;
      v = ld(&r, 0);
    }
    ss = fmaf(v, v, ss);
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)n + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const T t = rnd<T>(ld(xr, i) * r);        // (x * rsqrt(mean + eps)).to(dtype)
    hr[i] = rnd<T>(ld(&t, 0) * ld(w, i));     // ... * weight
  }
}

// Thread per element of qkv (1, (H + 2 KVH) hd): q -> q_out, k -> k_cache[pos],
// v -> v_cache[pos].  Rotate-half rotary embedding with fp32 tables (max_len, hd).
template <typename T>
__global__ void rope_append_kernel(const T* qkv, int nq, int nk, int hd, const float* cos_tab,
                                   const float* sin_tab, const int64_t* pos_p, T* q_out, T* k_cache,
                                   T* v_cache, int64_t tok_stride) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nq + 2 * nk) return;
  const int64_t pos = *pos_p;
  if (e >= nq + nk) {
    v_cache[pos * tok_stride + (e - nq - nk)] = qkv[e];
    return;
  }
  const int d = e % hd, half = hd / 2;
  const float x = ld(qkv, e);
  const float rot = d < half ? -ld(qkv, e + half) : ld(qkv, e - half);
  const float c = cos_tab[pos * hd + d], s = sin_tab[pos * hd + d];
  const T o = rnd<T>(__fadd_rn(__fmul_rn(x, c), __fmul_rn(rot, s)));
  if (e < nq) q_out[e] = o;
  else k_cache[pos * tok_stride + (e - nq)] = o;
}

// One CTA of 64 threads per query head.  Tail tokens [full, n) with
// n = pos + 1 and full = n rounded down to 64; the kernel state (m in log2
// units, l, unnormalised acc) of the whole tiles is merged by log-sum-exp.
template <typename T>
__global__ void tail_merge_kernel(const T* q, int group, int hd, const T* k_cache, const T* v_cache,
                                  int64_t tok_stride, int64_t max_len, const int64_t* pos_p, const float* m_in,
                                  const float* l_in, const float* acc_in, float scale_log2, T* out) {
  __shared__ float red[32];
  __shared__ float pt[64];
  __shared__ float qs[256];
  const int h = blockIdx.x, kvh = h / group, t = threadIdx.x;
  const int64_t n = *pos_p + 1, full = n - (n & 63);
  const int r = (int)(n - full);  // tail tokens
  for (int d = t; d < hd; d += blockDim.x) qs[d] = ld(q, (int64_t)h * hd + d);
  __syncthreads();
  float lg = -INFINITY;
  if (t < r) {
    const T* kr = k_cache + (full + t) * tok_stride + (int64_t)kvh * hd;
    float s = 0.f;
    if ((hd & 7) == 0 && ((reinterpret_cast<uintptr_t>(kr) & 15u) == 0)) {
      for (int d = 0; d < hd; d += 8) {  // 16-byte loads of the key row
        const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fmaf(qs[d + j], ld(e, j), s);
      }
    } else {
      for (int d = 0; d < hd; ++d) s = fmaf(qs[d], ld(kr, d), s);
    }
    lg = s * scale_log2;
  }
  const float mt = fmaxf(block_max(lg, red), -1e9f);  // an empty tail weighs 0
  const float p = exp2f(lg - mt);
  pt[t] = p;
  const float lt = block_sum(p, red);  // its barriers also publish pt
  // the state of the whole tiles comes from the kernel before this one (a
  // programmatic dependent launch: everything above overlapped it)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const float m0 = m_in[h], M = fmaxf(m0, mt);
  const float a = exp2f(m0 - M), b = exp2f(mt - M);
  const float L = fmaf(l_in[h], a, lt * b);
  for (int d = t; d < hd; d += blockDim.x) {
    const T* vc = v_cache + full * tok_stride + (int64_t)kvh * hd + d;
    float s = 0.f;
#pragma unroll 8
    for (int j = 0; j < r; ++j) s = fmaf(pt[j], ld(vc, (int64_t)j * tok_stride), s);
    out[(int64_t)h * hd + d] = rnd<T>(fmaf(acc_in[(int64_t)h * hd + d], a, s * b) / fmaxf(L, 1e-9f));
  }
}

inline int finish() { return cudaGetLastError() == cudaSuccess ? OC_OK : OC_ERR_CUDA; }

}  // namespace

extern "C" int oc_add_rms_norm(void* x, const void* y, const void* weight, void* h, int64_t rows, int64_t n,
                               float eps, int dtype, void* stream) {
  if (!x || !weight || !h || rows < 0 || n < 1) return OC_ERR_INVALID;
  if (rows == 0) return OC_OK;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == OC_BF16)
    add_rms_norm_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, st>>>(
        static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y),
        static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(h), n, eps);
  else if (dtype == OC_F16)
    add_rms_norm_kernel<__half><<<(unsigned)rows, 256, 0, st>>>(static_cast<__half*>(x), static_cast<const __half*>(y),
                                                                static_cast<const __half*>(weight),
                                                                static_cast<__half*>(h), n, eps);
  else
    return OC_ERR_UNSUPPORTED;
  return finish();
}

extern "C" int oc_rope_cache_append(const void* qkv, int heads, int kv_heads, int head_dim, const float* cos_tab,
                                    const float* sin_tab, const int64_t* pos, void* q_out, void* k_cache,
                                    void* v_cache, int64_t cache_token_stride, int dtype, void* stream) {
  if (!qkv || !cos_tab || !sin_tab || !pos || !q_out || !k_cache || !v_cache || heads < 1 || kv_heads < 1 ||
      head_dim < 2 || (head_dim & 1) || cache_token_stride < (int64_t)kv_heads * head_dim)
    return OC_ERR_INVALID;
  const int nq = heads * head_dim, nk = kv_heads * head_dim, tot = nq + 2 * nk;
  auto st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((tot + 255) / 256);
  if (dtype == OC_BF16)
    rope_append_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(qkv), nq, nk, head_dim, cos_tab, sin_tab, pos,
        static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), cache_token_stride);
  else if (dtype == OC_F16)
    rope_append_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(qkv), nq, nk, head_dim, cos_tab,
                                                     sin_tab, pos, static_cast<__half*>(q_out),
                                                     static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
                                                     cache_token_stride);
  else
    return OC_ERR_UNSUPPORTED;
  return finish();
}

extern "C" int oc_tail_merge(const void* q, int heads, int kv_heads, int head_dim, const void* k_cache,
                             const void* v_cache, int64_t cache_token_stride, int64_t max_len, const int64_t* pos,
                             const float* m, const float* l, const float* acc, float scale_log2, void* out,
                             int dtype, void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !m || !l || !acc || !out || heads < 1 || kv_heads < 1 ||
      heads % kv_heads || head_dim < 1 || head_dim > 256 || max_len < 1)
    return OC_ERR_INVALID;
  auto st = static_cast<cudaStream_t>(stream);
  const int group = heads / kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)heads);
  cfg.blockDim = dim3(64);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == OC_BF16)
    e = cudaLaunchKernelEx(&cfg, tail_merge_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(q), group,
                           head_dim, static_cast<const __nv_bfloat16*>(k_cache),
                           static_cast<const __nv_bfloat16*>(v_cache), cache_token_stride, max_len, pos, m, l, acc,
                           scale_log2, static_cast<__nv_bfloat16*>(out));
  else if (dtype == OC_F16)
    e = cudaLaunchKernelEx(&cfg, tail_merge_kernel<__half>, static_cast<const __half*>(q), group, head_dim,
                           static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
                           cache_token_stride, max_len, pos, m, l, acc, scale_log2, static_cast<__half*>(out));
  else
    return OC_ERR_UNSUPPORTED;
  if (e != cudaSuccess) return OC_ERR_CUDA;
  return finish();
}
