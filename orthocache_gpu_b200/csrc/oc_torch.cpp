// Compiled Python binding of the hot decode calls (V2 and V3).
//
// The ctypes path marshals ~30 arguments per call and reads tensor strides
// and pointers from Python, which costs more host time than a short decode
// takes on the GPU.  This module takes the tensors themselves, allocates the
// output with torch, and calls the library's C ABI
// (include/orthocache_b200.h) directly; it adds no GPU code.
#include <torch/extension.h>

#include <cstdint>

#include "../../include/orthocache_b200.h"

namespace {

int code_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return OC_F32;
    case at::kHalf: return OC_F16;
    case at::kBFloat16: return OC_BF16;
    case at::kFloat8_e4m3fn: return OC_F8E4M3;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check(int rc, const char* what) {
  TORCH_CHECK(rc == OC_OK, what, ": ", oc_status_string(rc), " (code ", rc, ")");
}

void* ptr_or_null(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// q (H, hd); keys / values (H, S, hd) with a contiguous last dim; returns out (H, hd) in out_dtype.
at::Tensor v2(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double zeta_max, int64_t num_splits,
              int64_t num_sms, at::ScalarType out_dtype, const c10::optional<at::Tensor>& mask,
              int64_t retained, int64_t status, int64_t ws, int64_t ws_bytes, int64_t stream) {
  const int64_t H = q.size(0), hd = q.size(1), S = k.size(1);
  at::Tensor out = at::empty({H, hd}, q.options().dtype(out_dtype));
  check(oc_fused_attention_v2(q.data_ptr(), code_of(q), q.stride(0), k.data_ptr(), code_of(k), k.stride(0),
                              k.stride(1), v.data_ptr(), code_of(v), v.stride(0), v.stride(1), (int)H, S, (int)hd,
                              zeta_max, (int)num_splits, (int)num_sms, out.data_ptr(), code_of(out), out.stride(0),
                              static_cast<uint8_t*>(ptr_or_null(mask)), reinterpret_cast<uint32_t*>(retained),
                              reinterpret_cast<uint32_t*>(status), reinterpret_cast<void*>(ws), (size_t)ws_bytes,
                              reinterpret_cast<void*>(stream)),
        "fused_orthocache_attention_v2");
  return out;
}

// q (B, Hq, hd); keys / values (B, KVH, S, hd); returns out (B, Hq, hd) in out_dtype.
at::Tensor v3(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double tau, int64_t group,
              int64_t num_splits, int64_t num_sms, at::ScalarType out_dtype, const c10::optional<at::Tensor>& mask,
              int64_t retained, int64_t status, int64_t ws, int64_t ws_bytes, int64_t stream) {
  const int64_t B = k.size(0), KVH = k.size(1), S = k.size(2), hd = k.size(3);
  at::Tensor out = at::empty({B, KVH * group, hd}, q.options().dtype(out_dtype));
  check(oc_fused_attention_v3_gqa(q.data_ptr(), code_of(q), q.stride(0), q.stride(1), k.data_ptr(), code_of(k),
                                  k.stride(0), k.stride(1), k.stride(2), v.data_ptr(), code_of(v), v.stride(0),
                                  v.stride(1), v.stride(2), (int)B, (int)KVH, (int)group, S, (int)hd, tau,
                                  (int)num_splits, (int)num_sms, out.data_ptr(), code_of(out), out.stride(0),
                                  out.stride(1), static_cast<uint8_t*>(ptr_or_null(mask)),
                                  reinterpret_cast<uint32_t*>(retained), reinterpret_cast<uint32_t*>(status),
                                  reinterpret_cast<void*>(ws), (size_t)ws_bytes, reinterpret_cast<void*>(stream)),
        "fused_orthocache_attention_v3_gqa");
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "compiled binding of the V2 / V3 decode calls of liborthocache_b200";
  m.def("v2", &v2);
  m.def("v3", &v3);
}
