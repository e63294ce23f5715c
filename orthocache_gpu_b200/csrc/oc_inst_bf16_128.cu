#define OC_KT __nv_bfloat16
#define OC_KNAME bf16
#define OC_HEADDIM 128
#define OC_VTYPES(X) X(2, __nv_bfloat16)
#include "oc_inst.cuh"
