#define OC_KT __nv_fp8_e4m3
#define OC_KNAME f8
#define OC_HEADDIM 32
#define OC_VTYPES(X) X(1, __half) X(2, __nv_bfloat16) X(0, float)
#include "oc_inst.cuh"
