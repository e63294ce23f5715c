#define OC_KT float
#define OC_KNAME f32
#define OC_HEADDIM 32
#define OC_VTYPES(X) X(0, float)
#include "oc_inst.cuh"
