// Explicit instantiation of the decode kernel for one key dtype.  Included by
// oc_inst_<dtype>_<hd>.cu with OC_KT (key type), OC_KNAME (suffix), OC_HEADDIM and
// OC_VTYPES(X) (the value types compiled with that key type) defined, so the
// instantiations compile as separate translation units in parallel.
#include "oc_decode.cuh"
#include "oc_dispatch.h"

namespace oc {

#define OC_CAT2(a, b) a##b
#define OC_CAT(a, b) OC_CAT2(a, b)

#ifndef OC_SLOTS
#define OC_SLOTS 3
#endif
constexpr int kSlots = OC_SLOTS;  // per-warp ring depth

template <typename VT, int HD, bool TC>
static cudaError_t launch_gc_tc(const DecodeParams& p, const TensorMaps& m, int gc, bool attn, int sms,
                                cudaStream_t st) {
  if (!attn) return launch_decode<OC_KT, OC_KT, HD, 1, false, kSlots, TC>(p, m.k, m.v, sms, st);
  switch (gc) {
    case 1: return launch_decode<OC_KT, VT, HD, 1, true, kSlots, TC>(p, m.k, m.v, sms, st);
    case 2: return launch_decode<OC_KT, VT, HD, 2, true, kSlots, TC>(p, m.k, m.v, sms, st);
    case 4: return launch_decode<OC_KT, VT, HD, 4, true, kSlots, TC>(p, m.k, m.v, sms, st);
    default: return launch_decode<OC_KT, VT, HD, 8, true, kSlots, TC>(p, m.k, m.v, sms, st);
  }
}

// tensor-core path: 16-bit keys with values of the same type, head_dim >= 64
template <typename VT, int HD>
static cudaError_t launch_gc(const DecodeParams& p, const TensorMaps& m, int gc, bool attn, int sms,
                             cudaStream_t st, bool tc) {
  constexpr bool kTcOk = sizeof(OC_KT) == 2 && std::is_same<VT, OC_KT>::value && HD >= 64;
  if constexpr (kTcOk) {
    if (tc) return launch_gc_tc<VT, HD, true>(p, m, gc, attn, sms, st);
  }
  return launch_gc_tc<VT, HD, false>(p, m, gc, attn, sms, st);
}

// One head_dim per translation unit (OC_HEADDIM): int dispatch_<kname>_<hd>(...)
int OC_CAT(OC_CAT(OC_CAT(dispatch_, OC_KNAME), _), OC_HEADDIM)(const DecodeParams& p, const TensorMaps& m, int v_dtype,
                                                              int gc, bool attn, int sms, cudaStream_t st, bool tc) {
#define OC_CASE(code, VT)                                                 \
  if (v_dtype == code || !attn) {                                         \
    const cudaError_t e = launch_gc<VT, OC_HEADDIM>(p, m, gc, attn, sms, st, tc);     \
    return e == cudaSuccess ? 0 : 4;                                      \
  }
  OC_VTYPES(OC_CASE)
#undef OC_CASE
  return 2;
}

}  // namespace oc
