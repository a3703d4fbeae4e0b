// eval_f64.cu — fp64 instantiations of the fused evaluation kernel (fp64 fits and the
// fp64 audit of fp32 fits).
#define CUSR_T double
#define CUSR_FN(name) name##_f64
#define CUSR_KCS(X) X(1) X(2) X(4) X(8) X(32)
#include "eval_inst.cuh"
