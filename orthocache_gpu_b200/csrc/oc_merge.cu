// Stand-alone log-sum-exp merge of partial softmax states (the split-K
// reduction of fused_eviction.py:316-373 as its own kernel).  Used to combine
// the per-GPU partials of a sequence-sharded decode.
#include <cmath>

#include "../../include/orthocache_b200.h"
#include "oc_decode.cuh"

namespace {

__global__ void lse_merge_kernel(const float* __restrict__ m, const float* __restrict__ l,
                                 const float* __restrict__ acc, int parts, int hd, void* out, int out_dtype) {
  const int64_t u = blockIdx.x;
  const float* mu = m + u * parts;
  const float* lu = l + u * parts;
  float M = -INFINITY;
  for (int p = 0; p < parts; ++p) M = fmaxf(M, mu[p]);
  float lt = 0.f;
  for (int p = 0; p < parts; ++p) lt = fmaf(lu[p], exp2f(mu[p] - M), lt);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float a = 0.f;
    for (int p = 0; p < parts; ++p) a = fmaf(acc[(u * parts + p) * hd + d], exp2f(mu[p] - M), a);
    oc::store_any(out, u * hd + d, out_dtype, a / fmaxf(lt, 1e-9f));
  }
}

}  // namespace

extern "C" int oc_lse_merge(const float* m, const float* l, const float* acc, int64_t num_units, int num_parts,
                            int head_dim, void* out, int out_dtype, void* stream) {
  if (!m || !l || !acc || !out || num_units < 0 || num_parts < 1 || head_dim < 1 || head_dim > 1024)
    return OC_ERR_INVALID;
  if (out_dtype != OC_F32 && out_dtype != OC_F16 && out_dtype != OC_BF16) return OC_ERR_UNSUPPORTED;
  if (num_units == 0) return OC_OK;
  const int threads = head_dim < 32 ? 32 : head_dim;
  lse_merge_kernel<<<(unsigned)num_units, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      m, l, acc, num_parts, head_dim, out, out_dtype);
  return cudaGetLastError() == cudaSuccess ? OC_OK : OC_ERR_CUDA;
}
