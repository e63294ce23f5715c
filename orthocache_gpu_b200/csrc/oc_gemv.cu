// GEMV of one decode token for the model driver (model.py): out[n] =
// sum_k h[k] W[n, k], W in the (out_features, in_features) layout of a
// linear layer (row n contiguous, leading dimension ldw), 16-bit weights and
// activations, fp32 accumulation.  A decode step of a TinyLlama-shaped model
// reads about 2 GB of weights per token through five such products per
// layer; each is HBM-bound, so the kernel's job is to stream W's rows with
// long contiguous reads and enough bytes in flight on every SM.
//
//   Persistent grid (one wave of resident CTAs of 16 warps); each warp takes
//   PAIRS of output rows in turn and reads both rows in 2048-column pieces:
//   lane l loads 16 bytes at columns 8 (l + 32 i), i < 8, of each row (16
//   loads of 16 bytes in flight per lane, 4 KB contiguous per row and piece),
//   then a butterfly reduction gives the two dot products (with few pairs
//   and K > 2048, two or four warps of a CTA share a pair, one piece each in
//   turn, and add their sums through shared memory).  The pair is
//   what the epilogues need together:
//     PLAIN     rows (2p, 2p+1)          out[n] = round(sum_n)
//     SILU_MUL  rows (2j, 2j+1) = (a_j, b_j), W's rows interleaved
//               out[j] = round(round(silu(round(a_j))) * round(b_j))
//               (the PyTorch ops F.silu(a) * b on 16-bit tensors)
//     ROPE      rows (d, d + hd/2) of one head of the q | k | v projection:
//               rotate-half rotary embedding of q and k at position *pos
//               (fp32 tables); q to q_out, k and v appended to the
//               token-major caches (the arithmetic of oc_rope_cache_append)
//
// Prologue (norm_w != NULL): v = round(x + y) (y optional), written to x_out
// by CTA 0, and h = round(round(v * rsqrt(mean(v^2) + eps)) * norm_w): the
// residual add + RMSNorm of the block input, recomputed by every CTA from the
// 2 K input values (L2-resident), so no normalisation launch sits between
// the blocks.  x_out must not alias x or y.
//
// Each launch is a programmatic dependent of the kernel before it on the
// stream: CTAs are scheduled while that kernel drains, and wait for it
// (griddepcontrol.wait) before reading the activations.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>

#include "../../include/orthocache_b200.h"

namespace {

constexpr int kWarps = 16;
constexpr int kMaxK = 8192;   // activations held in shared memory (fp32)
constexpr int kPiece = 2048;  // columns of a row read per pass (32 lanes x 8 loads x 8)

enum { EPI_PLAIN = 0, EPI_SILU_MUL = 1, EPI_ROPE = 2 };

template <typename T>
struct Cvt;
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 r(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ float f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half r(float x) { return __float2half_rn(x); }
};
template <typename T>
__device__ __forceinline__ float rf(float x) {  // round to T and back
  return Cvt<T>::f(Cvt<T>::r(x));
}

struct RopeArgs {
  int nq, nk, hd;
  const float* cos_tab;
  const float* sin_tab;
  const int64_t* pos;
  void* q_out;
  void* k_cache;
  void* v_cache;
  int64_t tok_stride;
};

template <typename T, int EPI>
__global__ void __launch_bounds__(32 * kWarps) gemv_kernel(const T* __restrict__ x, const T* __restrict__ y,
                                                          const T* __restrict__ norm_w, float eps,
                                                          T* __restrict__ x_out, const T* __restrict__ W,
                                                          int64_t ldw, int K, int N, int S,
                                                          T* __restrict__ out, RopeArgs ra) {
  __shared__ __align__(16) float hs[kMaxK];
  __shared__ float wsum[kWarps];
  __shared__ float2 part[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int npairs = N / 2;
  // S warps share a pair (S = 1, 2 or 4): warp `sub` of the group reads pieces sub, sub + S, ...
  const int sub = warp % S, slot = warp / S, slots = kWarps / S;
  const int64_t gw = (int64_t)blockIdx.x * slots + slot, nw = (int64_t)gridDim.x * slots;

  // rows of pair p
  auto rows = [&](int p, int& r0, int& r1) {
    if (EPI == EPI_ROPE) {
      const int half = ra.hd / 2, base = (p / half) * ra.hd, d = p % half;
      r0 = base + d;
      r1 = base + d + half;
    } else {
      r0 = 2 * p;
      r1 = 2 * p + 1;
    }
  };
  uint4 w0[8], w1[8];
  auto load_piece = [&](int p, int k0) {
    int r0, r1;
    rows(p, r0, r1);
    const T* a = W + (int64_t)r0 * ldw + k0;
    const T* b = W + (int64_t)r1 * ldw + k0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = 8 * (lane + 32 * i);
      if (k0 + k < K) {
        w0[i] = __ldcs(reinterpret_cast<const uint4*>(a + k));
        w1[i] = __ldcs(reinterpret_cast<const uint4*>(b + k));
      } else {
        w0[i] = w1[i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  // the first pair's first piece goes out before the activations are read
  int p = (int)gw;
  const int kfirst = sub * kPiece;
  if (p < npairs && kfirst < K) load_piece(p, kfirst);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (norm_w) {
    float ss = 0.f;
    for (int k8 = tid * 8; k8 < K; k8 += 32 * kWarps * 8) {  // K % 8 == 0, 16-byte aligned rows
      const uint4 xr = *reinterpret_cast<const uint4*>(x + k8);
      uint4 yr = make_uint4(0u, 0u, 0u, 0u);
      if (y) yr = *reinterpret_cast<const uint4*>(y + k8);
      const T* xe = reinterpret_cast<const T*>(&xr);
      const T* ye = reinterpret_cast<const T*>(&yr);
      uint4 vr;
      T* ve = reinterpret_cast<T*>(&vr);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v = Cvt<T>::f(xe[j]);
        if (y) v = rf<T>(v + Cvt<T>::f(ye[j]));
        ve[j] = Cvt<T>::r(v);
        hs[k8 + j] = v;
        ss = fmaf(v, v, ss);
      }
      if (x_out && blockIdx.x == 0) *reinterpret_cast<uint4*>(x_out + k8) = vr;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) wsum[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += wsum[i];
    const float r = rsqrtf(tot / (float)K + eps);
    for (int k = tid; k < K; k += 32 * kWarps) hs[k] = rf<T>(rf<T>(hs[k] * r) * Cvt<T>::f(norm_w[k]));
  } else {
    for (int k = tid; k < K; k += 32 * kWarps) hs[k] = Cvt<T>::f(x[k]);
  }
  __syncthreads();

  for (; p < npairs; p += (int)nw) {
    float s0 = 0.f, s1 = 0.f;
    for (int k0 = kfirst; k0 < K; k0 += S * kPiece) {
      if (k0 > kfirst) load_piece(p, k0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = k0 + 8 * (lane + 32 * i);
        if (k < K) {
          const T* e0 = reinterpret_cast<const T*>(&w0[i]);
          const T* e1 = reinterpret_cast<const T*>(&w1[i]);
          const float4 ha = *reinterpret_cast<const float4*>(hs + k);
          const float4 hb = *reinterpret_cast<const float4*>(hs + k + 4);
          const float h[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            s0 = fmaf(h[j], Cvt<T>::f(e0[j]), s0);
            s1 = fmaf(h[j], Cvt<T>::f(e1[j]), s1);
          }
        }
      }
    }
    if (p + nw < npairs && kfirst < K) load_piece((int)(p + nw), kfirst);  // next pair, before the reduction
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (S > 1) {  // the group's partial sums, added in piece order by its first warp
      if (lane == 0) part[warp] = make_float2(s0, s1);
      asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(32 * S) : "memory");
      if (sub == 0) {
        s0 = 0.f;
        s1 = 0.f;
        for (int j = 0; j < S; ++j) {
          s0 += part[warp + j].x;
          s1 += part[warp + j].y;
        }
      }
      asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(32 * S) : "memory");
      if (sub != 0) continue;
    }
    if (lane != 0) continue;
    int r0, r1;
    rows(p, r0, r1);
    if (EPI == EPI_PLAIN) {
      out[r0] = Cvt<T>::r(s0);
      out[r1] = Cvt<T>::r(s1);
    } else if (EPI == EPI_SILU_MUL) {
      const float a = rf<T>(s0), b = rf<T>(s1);
      const float sa = rf<T>(a / (1.f + expf(-a)));
      out[p] = Cvt<T>::r(sa * b);
    } else {
      const int64_t pos = *ra.pos;
      const float v0 = rf<T>(s0), v1 = rf<T>(s1);
      if (r0 >= ra.nq + ra.nk) {
        T* vc = static_cast<T*>(ra.v_cache) + pos * ra.tok_stride - ra.nq - ra.nk;
        vc[r0] = Cvt<T>::r(v0);
        vc[r1] = Cvt<T>::r(v1);
      } else {
        const int d = r0 % ra.hd, h2 = ra.hd / 2;  // r1 = r0 + hd / 2
        const float c0 = ra.cos_tab[pos * ra.hd + d], n0 = ra.sin_tab[pos * ra.hd + d];
        const float c1 = ra.cos_tab[pos * ra.hd + d + h2], n1 = ra.sin_tab[pos * ra.hd + d + h2];
        const T o0 = Cvt<T>::r(__fadd_rn(__fmul_rn(v0, c0), __fmul_rn(-v1, n0)));
        const T o1 = Cvt<T>::r(__fadd_rn(__fmul_rn(v1, c1), __fmul_rn(v0, n1)));
        if (r0 < ra.nq) {
          static_cast<T*>(ra.q_out)[r0] = o0;
          static_cast<T*>(ra.q_out)[r1] = o1;
        } else {
          T* kc = static_cast<T*>(ra.k_cache) + pos * ra.tok_stride - ra.nq;
          kc[r0] = o0;
          kc[r1] = o1;
        }
      }
    }
  }
}

int sms() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

template <typename T, int EPI>
int launch(const void* x, const void* y, const void* norm_w, float eps, void* x_out, const void* W, int64_t ldw,
           int64_t K, int64_t N, void* out, const RopeArgs& ra, cudaStream_t st) {
  const int64_t npairs = N / 2;
  // persistent: every CTA resident at once (one wave)
  static int per_sm[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = dev >= 0 && dev < 64 ? per_sm[dev] : 0;
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<T, EPI>, 32 * kWarps, 0) != cudaSuccess ||
        occ < 1)
      occ = 1;
    if (dev >= 0 && dev < 64) per_sm[dev] = occ;
  }
  // warps per pair: enough pair tasks for every resident warp, at most one per 2048-column piece
  const int64_t warps = (int64_t)occ * sms() * kWarps, pieces = (K + kPiece - 1) / kPiece;
  int S = 1;
  while (S < 4 && 2 * S <= pieces && npairs * S < warps) S *= 2;
  const int64_t slots = kWarps / S;
  int64_t grid = (npairs + slots - 1) / slots;
  if (grid > (int64_t)occ * sms()) grid = (int64_t)occ * sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(32 * kWarps);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gemv_kernel<T, EPI>, static_cast<const T*>(x), static_cast<const T*>(y),
                         static_cast<const T*>(norm_w), eps, static_cast<T*>(x_out), static_cast<const T*>(W), ldw,
                         (int)K, (int)N, S, static_cast<T*>(out), ra) != cudaSuccess)
    return OC_ERR_CUDA;
  return OC_OK;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(const void* x, const void* y, const void* norm_w, const void* x_out, const void* W, int64_t ldw,
                 int64_t K, int64_t N) {
  if (!x || !W || K < 8 || K % 8 || K > kMaxK || N < 2 || N % 2 || N > (1 << 30) || ldw < K || ldw % 8 || !a16(W))
    return OC_ERR_INVALID;
  if (norm_w && (!a16(x) || (y && !a16(y)) || (x_out && !a16(x_out)))) return OC_ERR_INVALID;
  if (x_out && (x_out == x || (y && x_out == y))) return OC_ERR_INVALID;
  return OC_OK;
}

template <int EPI>
int dispatch(int dtype, const void* x, const void* y, const void* norm_w, float eps, void* x_out, const void* W,
             int64_t ldw, int64_t K, int64_t N, void* out, const RopeArgs& ra, void* stream) {
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == OC_BF16) return launch<__nv_bfloat16, EPI>(x, y, norm_w, eps, x_out, W, ldw, K, N, out, ra, st);
  if (dtype == OC_F16) return launch<__half, EPI>(x, y, norm_w, eps, x_out, W, ldw, K, N, out, ra, st);
  return OC_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" int oc_gemv(const void* x, const void* y, const void* norm_w, float eps, void* x_out, const void* W,
                       int64_t ldw, int64_t K, int64_t N, void* out, int epilogue, int dtype, void* stream) {
  const int rc = check_common(x, y, norm_w, x_out, W, ldw, K, N);
  if (rc != OC_OK) return rc;
  if (!out) return OC_ERR_INVALID;
  RopeArgs ra{};
  if (epilogue == OC_GEMV_PLAIN)
    return dispatch<EPI_PLAIN>(dtype, x, y, norm_w, eps, x_out, W, ldw, K, N, out, ra, stream);
  if (epilogue == OC_GEMV_SILU_MUL)
    return dispatch<EPI_SILU_MUL>(dtype, x, y, norm_w, eps, x_out, W, ldw, K, N, out, ra, stream);
  return OC_ERR_INVALID;
}

extern "C" int oc_gemv_qkv_rope(const void* x, const void* y, const void* norm_w, float eps, void* x_out,
                                const void* W, int64_t ldw, int64_t K, int heads, int kv_heads, int head_dim,
                                const float* cos_tab, const float* sin_tab, const int64_t* pos, void* q_out,
                                void* k_cache, void* v_cache, int64_t cache_token_stride, int dtype, void* stream) {
  if (heads < 1 || kv_heads < 1 || head_dim < 2 || (head_dim & 1) || !cos_tab || !sin_tab || !pos || !q_out ||
      !k_cache || !v_cache || cache_token_stride < (int64_t)kv_heads * head_dim)
    return OC_ERR_INVALID;
  const int64_t N = (int64_t)(heads + 2 * kv_heads) * head_dim;
  const int rc = check_common(x, y, norm_w, x_out, W, ldw, K, N);
  if (rc != OC_OK) return rc;
  RopeArgs ra{heads * head_dim, kv_heads * head_dim, head_dim, cos_tab, sin_tab, pos,
              q_out,            k_cache,             v_cache,  cache_token_stride};
  return dispatch<EPI_ROPE>(dtype, x, y, norm_w, eps, x_out, W, ldw, K, N, q_out, ra, stream);
}
