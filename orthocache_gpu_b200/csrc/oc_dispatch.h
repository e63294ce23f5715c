// Launch dispatchers, one translation unit per (key dtype, head_dim).
// Return 0 on success, 2 when the combination is not compiled, 4 on a
// launch error.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cuda.h>
#include <cstdint>

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
// Decode gate from cached key norms (oc_normcache.cu).
struct GateArgs {
  const void* q;
  int q_dtype;
  int64_t q_seq_stride, q_head_stride;
  int num_seqs, num_kv_heads, group, head_dim;
  const float* norms;
  int64_t norm_seq_stride, norm_head_stride;
  int num_tiles, max_tiles;
  float thr;  // float32(tau * 64 * head_dim)
  int tight, low_band, stat_median;
  uint8_t* evict;  // nullable, (num_seqs*num_kv_heads, evict_stride)
  int64_t evict_stride;
  float* q_norms;  // nullable, num_seqs*num_kv_heads
  int* list;       // nullable, (num_seqs*num_kv_heads, list_stride)
  int64_t list_stride;
  int* count;      // with list
};
int launch_decode_gate(const GateArgs& a, cudaStream_t st);
int launch_tile_high_norms(const void* keys, int k_dtype, int num_heads, int tiles, int hd, int64_t head_stride,
                           int64_t tok_stride, int hs, int he, float* out, int64_t out_stride, cudaStream_t st);
}  // namespace oc
