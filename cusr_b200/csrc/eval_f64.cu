// eval_f64.cu — fp64 instantiations of the fused evaluation kernel (fp64 fits and the
// fp64 audit of fp32 fits).
#include "launch.h"

namespace cusr {

namespace {

template <int KC, bool G>
cudaError_t one(const EvalParams<double> &p, int grid, size_t smem, cudaStream_t s) {
    lm_eval_kernel<double, EVAL_V, KC, G><<<grid, EVAL_THREADS, smem, s>>>(p);
    return cudaGetLastError();
}
template <int KC, bool G> int occ(size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, lm_eval_kernel<double, EVAL_V, KC, G>,
                                                      EVAL_THREADS, smem) != cudaSuccess)
        return 0;
    return n;
}
// dynamic shared memory limit = the device's opt-in maximum minus the kernel's static part
template <int KC, bool G> cudaError_t prep() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, lm_eval_kernel<double, EVAL_V, KC, G>);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lm_eval_kernel<double, EVAL_V, KC, G>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                optin - (int)fa.sharedSizeBytes);
}
}  // namespace

cudaError_t eval_launch_f64(int kc, bool grad, const EvalParams<double> &p, int grid, size_t smem,
                            cudaStream_t s) {
    if (!grad) return one<4, false>(p, grid, smem, s);
    switch (kc) {
        case 4: return one<4, true>(p, grid, smem, s);
        case 8: return one<8, true>(p, grid, smem, s);
        case 32: return one<32, true>(p, grid, smem, s);
        default: return cudaErrorInvalidValue;
    }
}

size_t eval_smem_f64(int kc, int code_cap, int n_vars, int spill_cap, int tape_cap) {
    switch (kc) {
        case 4: return EvalSmem<double, EVAL_V, 4>(code_cap, n_vars, spill_cap, tape_cap).total;
        case 8: return EvalSmem<double, EVAL_V, 8>(code_cap, n_vars, spill_cap, tape_cap).total;
        case 32: return EvalSmem<double, EVAL_V, 32>(code_cap, n_vars, spill_cap, tape_cap).total;
        default: return 0;
    }
}

int eval_blocks_per_sm_f64(int kc, bool grad, size_t smem) {
    if (!grad) return occ<4, false>(smem);
    switch (kc) {
        case 4: return occ<4, true>(smem);
        case 8: return occ<8, true>(smem);
        case 32: return occ<32, true>(smem);
        default: return 0;
    }
}

cudaError_t eval_prepare_f64() {
    cudaError_t e;
    if ((e = prep<4, false>()) != cudaSuccess) return e;
    if ((e = prep<4, true>()) != cudaSuccess) return e;
    if ((e = prep<8, true>()) != cudaSuccess) return e;
    return prep<32, true>();
}

}  // namespace cusr
