// launch.h — host-side launchers of the templated evaluation kernels (one translation unit
// per arithmetic type so the instantiations compile in parallel).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include "eval_kernel.cuh"

namespace cusr {

#ifndef CUSR_EVAL_V
#define CUSR_EVAL_V 2
#endif
#ifndef CUSR_EVAL_NT
#define CUSR_EVAL_NT 128
#endif
constexpr int EVAL_V = CUSR_EVAL_V;    // samples per thread (both precisions)
constexpr int EVAL_NT = CUSR_EVAL_NT;  // threads per block
constexpr int EVAL_THREADS = EVAL_NT;
// wide instantiations (twice the threads per block) for bins of long programs / large tapes
constexpr int EVAL_NT_WIDE = 2 * EVAL_NT;
// sample granularity of the input layout and of the work chunks: one round of a wide block
constexpr int EVAL_ROUND = EVAL_NT_WIDE * EVAL_V;

// kc: constant-count class (4, 8, 12, 16, 32 for fp32; 4, 8, 32 for fp64).
// grad = false launches the value-only kernel (lm_value_kernel: the fp64 audit and the
// finite-difference value passes); tg = reverse tape in global scratch (EvalParams::tape_g)
// instead of shared memory.
// wide = EVAL_NT_WIDE threads per block (grad launches only)
cudaError_t eval_launch_f32(int kc, bool grad, bool tg, bool wide, const EvalParams<float> &p,
                            int grid, size_t smem, cudaStream_t s);
cudaError_t eval_launch_f32_fast(int kc, bool grad, bool tg, bool wide, const EvalParams<float> &p,
                                 int grid, size_t smem, cudaStream_t s);
cudaError_t eval_launch_f64(int kc, bool grad, bool tg, bool wide, const EvalParams<double> &p,
                            int grid, size_t smem, cudaStream_t s);
size_t eval_smem_f32(int kc, int code_cap, int n_vars, int spill_cap, int tape_cap, bool tape_in_smem,
                     bool wide);
size_t eval_smem_f64(int kc, int code_cap, int n_vars, int spill_cap, int tape_cap, bool tape_in_smem,
                     bool wide);
// resident blocks per SM of an instantiation at the given dynamic shared memory
int eval_blocks_per_sm_f32(int kc, bool grad, bool tg, bool wide, size_t smem);
int eval_blocks_per_sm_f32_fast(int kc, bool grad, bool tg, bool wide, size_t smem);
int eval_blocks_per_sm_f64(int kc, bool grad, bool tg, bool wide, size_t smem);
// raise the dynamic shared-memory limit of every instantiation (once per device)
cudaError_t eval_prepare_f32();
cudaError_t eval_prepare_f32_fast();
cudaError_t eval_prepare_f64();

template <typename T> struct Launch;
// `fast` selects the --use_fast_math instantiations (fp32 only; ignored for fp64); `wide` the
// EVAL_NT_WIDE-thread ones. The shared-memory layout does not depend on `fast`.
template <> struct Launch<float> {
    static cudaError_t eval(int kc, bool g, bool tg, bool fast, bool wide, const EvalParams<float> &p,
                            int grid, size_t sm, cudaStream_t s) {
        return fast ? eval_launch_f32_fast(kc, g, tg, wide, p, grid, sm, s)
                    : eval_launch_f32(kc, g, tg, wide, p, grid, sm, s);
    }
    static size_t smem(int kc, int a, int b, int c, int d, bool ts, bool wide) {
        return eval_smem_f32(kc, a, b, c, d, ts, wide);
    }
    static int occ(int kc, bool g, bool tg, bool fast, bool wide, size_t sm) {
        return fast ? eval_blocks_per_sm_f32_fast(kc, g, tg, wide, sm)
                    : eval_blocks_per_sm_f32(kc, g, tg, wide, sm);
    }
};
template <> struct Launch<double> {
    static cudaError_t eval(int kc, bool g, bool tg, bool, bool wide, const EvalParams<double> &p,
                            int grid, size_t sm, cudaStream_t s) {
        return eval_launch_f64(kc, g, tg, wide, p, grid, sm, s);
    }
    static size_t smem(int kc, int a, int b, int c, int d, bool ts, bool wide) {
        return eval_smem_f64(kc, a, b, c, d, ts, wide);
    }
    static int occ(int kc, bool g, bool tg, bool, bool wide, size_t sm) {
        return eval_blocks_per_sm_f64(kc, g, tg, wide, sm);
    }
};

}  // namespace cusr
