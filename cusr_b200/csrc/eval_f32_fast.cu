// eval_f32_fast.cu — fp32 instantiations with the reference kernel's numerics: this file is
// compiled with --use_fast_math (the flags of cusr/kernel/Makefile:9), so sinf / cosf /
// expf / logf / powf map to the hardware approximations, division and square root are the
// approximate forms and denormals are flushed to zero.
#define CUSR_T float
#define CUSR_FN(name) name##_f32_fast
#define CUSR_KCS(X) X(1) X(2) X(4) X(8) X(12) X(16) X(32)
#define CUSR_FAST 1
#include "eval_inst.cuh"
