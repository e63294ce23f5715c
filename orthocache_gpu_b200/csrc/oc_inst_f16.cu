#define OC_KT __half
#define OC_KNAME f16
#define OC_MAX_HD 256
#define OC_VTYPES(X) X(1, __half)
#include "oc_inst.cuh"
