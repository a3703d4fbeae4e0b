/* cusr_debug.h — host-only helpers of libcusr_b200.so for testing the bytecode compiler
 * without a GPU. Not part of the drop-in surface (no counterpart in the reference). */
#ifndef CUSR_DEBUG_H
#define CUSR_DEBUG_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Compile one prefix tree (n_nodes nodes, K constants, n_vars inputs) into at most `cap`
 * program words: the forward program, the reverse program, then the row table ((K + 4) / 4
 * words: the tape slot of each gradient row and of the residual row, one byte each).
 * info_out[5] = {n_forward, n_spill, n_tape, unique_const, n_reverse}.
 * Returns CO_OK / CO_ERR_BOUNDS / CO_ERR_BADTREE / CO_ERR_NULLARG (cap too small). */
int cusr_compile_tree(const int32_t *nt, const float *nv, const int32_t *ci, int n_nodes, int K,
                      int n_vars, uint32_t *code_out, int cap, int32_t *info_out);

/* Run a compiled program on the host in fp64 at one sample: returns the value, and writes
 * df/dc_k to grad[0..K) when grad is not NULL (same programs as the device; `bwd` points at
 * the reverse program, which the row table follows). */
double cusr_eval_program(const uint32_t *fwd, int n_fwd, const uint32_t *bwd, int n_bwd,
                         const double *x, const double *c, int K, double *grad);

/* The start points the engine generates for tree m (CoOptions.n_starts, start_seed), computed
 * on the host with the same formulas: out[s * K + k] for starts 0..S-1 of a tree whose c_init
 * is c0[0..K). */
void cusr_start_points(uint64_t seed, int64_t m, int S, int K, const float *c0, float *out);

#ifdef __cplusplus
}
#endif

#endif /* CUSR_DEBUG_H */
