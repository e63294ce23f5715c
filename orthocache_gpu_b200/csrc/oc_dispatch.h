// Per-key-dtype launch dispatchers (one translation unit each).
// Return 0 on success, 2 when the combination is not compiled, 4 on a
// launch error.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>

namespace oc {
struct DecodeParams;
int dispatch_f32(const DecodeParams& p, int v_dtype, int hd, int gc, bool attn, cudaStream_t st);
int dispatch_f16(const DecodeParams& p, int v_dtype, int hd, int gc, bool attn, cudaStream_t st);
int dispatch_bf16(const DecodeParams& p, int v_dtype, int hd, int gc, bool attn, cudaStream_t st);
int dispatch_f8(const DecodeParams& p, int v_dtype, int hd, int gc, bool attn, cudaStream_t st);
size_t workspace_header_bytes();
}  // namespace oc
