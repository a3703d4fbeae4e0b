// eval_inst.cuh — host launchers for the instantiations of lm_eval_kernel<T, ...> of one
// arithmetic type; included by eval_f32.cu / eval_f32_fast.cu / eval_f64.cu with CUSR_T, the
// launcher suffix CUSR_FN, the list of constant-count classes CUSR_KCS(X) and CUSR_FAST
// (1 in the translation unit compiled with --use_fast_math) defined.
#include "launch.h"

#ifndef CUSR_FAST
#define CUSR_FAST 0
#endif

namespace cusr {
namespace {

template <int KC, bool G, bool TG, int NT = EVAL_NT>
cudaError_t one(const EvalParams<CUSR_T> &p, int grid, size_t smem, cudaStream_t s) {
    lm_eval_kernel<CUSR_T, EVAL_V, NT, KC, G, TG, (CUSR_FAST != 0)><<<grid, NT, smem, s>>>(p);
    return cudaGetLastError();
}
// value-only pass (its own kernel; shared-memory layout of the KC = 4 class, one tape slot)
cudaError_t value_one(const EvalParams<CUSR_T> &p, int grid, size_t smem, cudaStream_t s) {
    lm_value_kernel<CUSR_T, EVAL_V, EVAL_NT, (CUSR_FAST != 0)><<<grid, EVAL_NT, smem, s>>>(p);
    return cudaGetLastError();
}
int value_occ(size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, lm_value_kernel<CUSR_T, EVAL_V, EVAL_NT, (CUSR_FAST != 0)>,
                                                      EVAL_NT, smem) != cudaSuccess)
        return 0;
    return n;
}
cudaError_t value_prep() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, lm_value_kernel<CUSR_T, EVAL_V, EVAL_NT, (CUSR_FAST != 0)>);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lm_value_kernel<CUSR_T, EVAL_V, EVAL_NT, (CUSR_FAST != 0)>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
}
template <int KC, bool G, bool TG, int NT = EVAL_NT> int occ(size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, lm_eval_kernel<CUSR_T, EVAL_V, NT, KC, G, TG, (CUSR_FAST != 0)>,
                                                      NT, smem) != cudaSuccess)
        return 0;
    return n;
}
// dynamic shared memory limit = the device's opt-in maximum minus the kernel's static part
template <int KC, bool G, bool TG, int NT = EVAL_NT> cudaError_t prep() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, lm_eval_kernel<CUSR_T, EVAL_V, NT, KC, G, TG, (CUSR_FAST != 0)>);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lm_eval_kernel<CUSR_T, EVAL_V, NT, KC, G, TG, (CUSR_FAST != 0)>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                optin - (int)fa.sharedSizeBytes);
}
}  // namespace

cudaError_t CUSR_FN(eval_launch)(int kc, bool grad, bool tg, bool wide, const EvalParams<CUSR_T> &p,
                                 int grid, size_t smem, cudaStream_t s) {
    if (!grad) return value_one(p, grid, smem, s);
#define X(KC)                                                                                  \
    if (kc == KC) {                                                                            \
        if (wide) return tg ? one<KC, true, true, EVAL_NT_WIDE>(p, grid, smem, s)              \
                            : one<KC, true, false, EVAL_NT_WIDE>(p, grid, smem, s);            \
        return tg ? one<KC, true, true>(p, grid, smem, s) : one<KC, true, false>(p, grid, smem, s); \
    }
    CUSR_KCS(X)
#undef X
    return cudaErrorInvalidValue;
}

size_t CUSR_FN(eval_smem)(int kc, int code_cap, int n_vars, int spill_cap, int tape_cap,
                          bool tape_in_smem, bool wide) {
#define X(KC)                                                                                     \
    if (kc == KC)                                                                                 \
        return wide ? EvalSmem<CUSR_T, EVAL_V, EVAL_NT_WIDE, KC>(code_cap, n_vars, spill_cap,     \
                                                                 tape_cap, tape_in_smem).total    \
                    : EvalSmem<CUSR_T, EVAL_V, EVAL_NT, KC>(code_cap, n_vars, spill_cap, tape_cap, \
                                                            tape_in_smem).total;
    CUSR_KCS(X)
#undef X
    return 0;
}

int CUSR_FN(eval_blocks_per_sm)(int kc, bool grad, bool tg, bool wide, size_t smem) {
    if (!grad) return value_occ(smem);
#define X(KC)                                                                        \
    if (kc == KC) {                                                                  \
        if (wide) return tg ? occ<KC, true, true, EVAL_NT_WIDE>(smem)                \
                            : occ<KC, true, false, EVAL_NT_WIDE>(smem);              \
        return tg ? occ<KC, true, true>(smem) : occ<KC, true, false>(smem);          \
    }
    CUSR_KCS(X)
#undef X
    return 0;
}

cudaError_t CUSR_FN(eval_prepare)() {
    cudaError_t e = value_prep();
    if (e != cudaSuccess) return e;
#define X(KC)                                                                       \
    if ((e = prep<KC, true, false>()) != cudaSuccess) return e;                      \
    if ((e = prep<KC, true, true>()) != cudaSuccess) return e;                       \
    if ((e = prep<KC, true, false, EVAL_NT_WIDE>()) != cudaSuccess) return e;        \
    if ((e = prep<KC, true, true, EVAL_NT_WIDE>()) != cudaSuccess) return e;
    CUSR_KCS(X)
#undef X
    return cudaSuccess;
}

}  // namespace cusr
