// Explicit instantiation of the decode kernel for one key dtype.  Included by
// oc_inst_<dtype>.cu with OC_KT (key type), OC_KNAME (suffix) and
// OC_VTYPES(X) (the value types compiled with that key type) defined, so the
// instantiations compile as separate translation units in parallel.
#include "oc_decode.cuh"
#include "oc_dispatch.h"

namespace oc {

#define OC_CAT2(a, b) a##b
#define OC_CAT(a, b) OC_CAT2(a, b)

template <typename VT, int HD>
static cudaError_t launch_gc(const DecodeParams& p, int gc, bool attn, cudaStream_t st) {
  if (!attn) return launch_decode<OC_KT, OC_KT, HD, 1, false>(p, st);
  switch (gc) {
    case 1: return launch_decode<OC_KT, VT, HD, 1, true>(p, st);
    case 2: return launch_decode<OC_KT, VT, HD, 2, true>(p, st);
    case 4: return launch_decode<OC_KT, VT, HD, 4, true>(p, st);
    default: return launch_decode<OC_KT, VT, HD, 8, true>(p, st);
  }
}

template <typename VT>
static int launch_hd(const DecodeParams& p, int hd, int gc, bool attn, cudaStream_t st) {
  cudaError_t e;
  switch (hd) {
#if OC_MAX_HD >= 16
    case 16: e = launch_gc<VT, 16>(p, gc, attn, st); break;
#endif
    case 32: e = launch_gc<VT, 32>(p, gc, attn, st); break;
    case 64: e = launch_gc<VT, 64>(p, gc, attn, st); break;
    case 128: e = launch_gc<VT, 128>(p, gc, attn, st); break;
#if OC_MAX_HD >= 256
    case 256: e = launch_gc<VT, 256>(p, gc, attn, st); break;
#endif
    default: return 2;
  }
  return e == cudaSuccess ? 0 : 4;
}

int OC_CAT(dispatch_, OC_KNAME)(const DecodeParams& p, int v_dtype, int hd, int gc, bool attn,
                                cudaStream_t st) {
#define OC_CASE(code, VT) \
  if (v_dtype == code || !attn) return launch_hd<VT>(p, hd, gc, attn, st);
  OC_VTYPES(OC_CASE)
#undef OC_CASE
  return 2;
}

}  // namespace oc
