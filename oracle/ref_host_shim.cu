// ref_host_shim.cu — TEST INFRASTRUCTURE ONLY. Compiled together with the reference's own
// interpreter headers (cusr/kernel/ad_interp.cuh, revad_interp.cuh) by oracle/Makefile, it
// exposes their host builds through a C ABI so the CPU tests can pin the oracle's value and
// Jacobian rules against the reference implementation itself.
#include "ad_interp.cuh"
#include "revad_interp.cuh"

extern "C" {

// value of one tree at one sample (ad_interp.cuh:281-329)
float ref_value(const int *nt, const float *nv, int n_nodes, const int *ci, const float *x,
                const float *c) {
    return eval_tree_val_host(nt, nv, n_nodes, ci, x, c);
}

// reverse-mode gradient, all K columns (revad_interp.cuh:66-157)
void ref_vjp(const int *nt, const float *nv, int n_nodes, const int *ci, const float *x,
             const float *c, int K, float *grad) {
    eval_tree_vjp_d(nt, nv, n_nodes, ci, x, c, K, grad);
}

// forward-mode value + tangents of columns [col_lo, col_lo + W) (ad_interp.cuh:58-233)
void ref_jvp(const int *nt, const float *nv, int n_nodes, const int *ci, const float *x,
             const float *c, int col_lo, int W, float *val, float *tangents) {
    eval_tree_jvp_d(nt, nv, n_nodes, ci, x, c, col_lo, W, val, tangents);
}

int ref_limits(int *max_stack, int *max_k, int *max_nodes) {
    *max_stack = MAX_STACK;
    *max_k = MAX_K;
    *max_nodes = MAX_NODES;
    return 0;
}

}
