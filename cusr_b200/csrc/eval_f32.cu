// eval_f32.cu — fp32 instantiations of the fused evaluation kernel (CO_PREC_FP32): the SFU
// arithmetic of ops.h (hardware reciprocal / square root / 2^x brought to about one ulp, own
// sin / cos reduction and polynomials). Building with -DCUSR_IEEE_F32 gives the IEEE library
// functions instead (for comparisons).
#ifndef CUSR_IEEE_F32
#define CUSR_SFU 1
#endif
#define CUSR_T float
#define CUSR_FN(name) name##_f32
#define CUSR_KCS(X) X(1) X(2) X(4) X(8) X(12) X(16) X(32)
#include "eval_inst.cuh"
