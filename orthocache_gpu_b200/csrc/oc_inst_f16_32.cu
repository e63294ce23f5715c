#define OC_KT __half
#define OC_KNAME f16
#define OC_HEADDIM 32
#define OC_VTYPES(X) X(1, __half)
#include "oc_inst.cuh"
