// eval_f32.cu — fp32 instantiations of the fused evaluation kernel.
#define CUSR_T float
#define CUSR_FN(name) name##_f32
#define CUSR_KCS(X) X(1) X(2) X(4) X(8) X(12) X(16) X(32)
#include "eval_inst.cuh"
