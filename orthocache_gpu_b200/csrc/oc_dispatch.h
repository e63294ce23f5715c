// Launch dispatchers, one translation unit per (key dtype, head_dim).
// Return 0 on success, 2 when the combination is not compiled, 4 on a
// launch error.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cuda.h>

namespace oc {
struct DecodeParams;
// TMA descriptors of the key and value tensors (unused when there is no tile)
struct TensorMaps {
  CUtensorMap k, v;
};
int dispatch_f32_16(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f32_32(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f32_64(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f32_128(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f16_16(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f16_32(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f16_64(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f16_128(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f16_256(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_bf16_16(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_bf16_32(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_bf16_64(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_bf16_128(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_bf16_256(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f8_16(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f8_32(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f8_64(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f8_128(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
int dispatch_f8_256(const DecodeParams& p, const TensorMaps& m, int v_dtype, int gc, bool attn, int num_sms, cudaStream_t st, bool tc);
}  // namespace oc
