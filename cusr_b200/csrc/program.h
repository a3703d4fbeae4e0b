// program.h — the compiled tree program executed by the device interpreter.
//
// The pop.bin bytecode (prefix order, one node per slot: nt/nv/ci, cusr/kernel/pop_format.h)
// is compiled on the host, once per call, into a short register-stack program:
//
//   * the value being built lives in a register ("TOS") of every thread;
//   * VAR and CONST leaves that feed a binary operator are folded into that operator as its
//     source operand (no push / pop);
//   * the two subtrees of a binary node are evaluated in Sethi–Ullman order (the one that
//     needs more stack first), so the spill stack in shared memory is as shallow as it can
//     be; the order of evaluation does not change any value (every node still computes
//     `left OP right` on the same operands, cusr/kernel/lm_core.cuh:85-101);
//   * each instruction carries the shared-memory slot of its spill (sd) and of its reverse-
//     mode tape entries (ts), so the forward and backward sweeps address the same words.
//
// Instruction word (32 bits):
//   [0,6)   op       OP_*
//   [6,8)   mode     source operand: M_POP (spill stack slot sd), M_VAR (x[idx]),
//                    M_CONST (c[idx]), M_NONE (unary)
//   [8]     swap     1: the source operand is the LEFT operand (src OP tos)
//   [9]     push     OP_LOAD only: spill the live TOS to slot sd before loading
//   [10,18) idx      variable index or constant rank
//   [18,24) sd       spill slot
//   [24,32) ts       first tape slot of this instruction
#pragma once
#include <stdint.h>

// host-only translation units (pack.cpp) see the CUDA qualifiers as no-ops
#if !defined(__CUDACC__)
#ifndef __host__
#define __host__
#endif
#ifndef __device__
#define __device__
#endif
#ifndef __forceinline__
#define __forceinline__ inline
#endif
#endif

namespace cusr {

enum Op : uint32_t {
    OP_LOAD = 0,
    // unary (value in TOS)
    OP_SIN = 1, OP_COS, OP_TAN, OP_SINH, OP_COSH, OP_TANH,
    OP_LOG, OP_LOGABS, OP_EXP, OP_INV, OP_NEG, OP_ABS, OP_SQRT, OP_SQRTABS, OP_UZERO,
    // binary (TOS OP src, or src OP TOS when swap)
    OP_ADD = 16, OP_SUB, OP_MUL, OP_DIV, OP_POW, OP_POWABS, OP_MAX, OP_MIN,
    OP_LT, OP_GT, OP_LE, OP_GE, OP_BZERO,
    OP_COUNT
};

enum Mode : uint32_t { M_POP = 0, M_VAR = 1, M_CONST = 2, M_NONE = 3 };

// pop.bin node types and EvoGP operator ids (cusr/kernel/ad_interp.cuh:21-31,
// cusr/benchmark/interp.py:18-29).
enum NodeType : int32_t { NT_VAR = 0, NT_CONST = 1, NT_UFUNC = 2, NT_BFUNC = 3 };
enum FuncId : int32_t {
    F_ADD = 1, F_SUB = 2, F_MUL = 3, F_DIV = 4, F_LOOSE_DIV = 5, F_POW = 6, F_LOOSE_POW = 7,
    F_MAX = 8, F_MIN = 9, F_LT = 10, F_GT = 11, F_LE = 12, F_GE = 13,
    F_SIN = 14, F_COS = 15, F_TAN = 16, F_SINH = 17, F_COSH = 18, F_TANH = 19,
    F_LOG = 20, F_LOOSE_LOG = 21, F_EXP = 22, F_INV = 23, F_LOOSE_INV = 24,
    F_NEG = 25, F_ABS = 26, F_SQRT = 27, F_LOOSE_SQRT = 28
};

__host__ __device__ constexpr inline uint32_t enc(uint32_t op, uint32_t mode, uint32_t swap,
                                                  uint32_t push, uint32_t idx, uint32_t sd,
                                                  uint32_t ts) {
    return (op & 63u) | ((mode & 3u) << 6) | ((swap & 1u) << 8) | ((push & 1u) << 9) |
           ((idx & 255u) << 10) | ((sd & 63u) << 18) | ((ts & 255u) << 24);
}
__host__ __device__ inline uint32_t w_op(uint32_t w)   { return w & 63u; }
__host__ __device__ inline uint32_t w_mode(uint32_t w) { return (w >> 6) & 3u; }
__host__ __device__ inline uint32_t w_swap(uint32_t w) { return (w >> 8) & 1u; }
__host__ __device__ inline uint32_t w_push(uint32_t w) { return (w >> 9) & 1u; }
__host__ __device__ inline uint32_t w_idx(uint32_t w)  { return (w >> 10) & 255u; }
__host__ __device__ inline uint32_t w_sd(uint32_t w)   { return (w >> 18) & 63u; }
__host__ __device__ inline uint32_t w_ts(uint32_t w)   { return (w >> 24) & 255u; }

constexpr int PROG_MAX_SPILL = 63;   // sd field
constexpr int PROG_MAX_TAPE  = 255;  // ts field (+1 for two-slot entries)

// Per-tree descriptor uploaded to the device (48 bytes).
struct TreeDesc {
    int32_t code_off;    // first instruction in the code array
    int32_t n_instr;
    int32_t K;           // constants of the tree
    int32_t c_off;       // offset of the tree's constants
    int64_t y_off;       // element offset of the tree's target row (0 when shared)
    int64_t p_off;       // element offset of the tree's per-chunk partial sums
    int64_t q_off;       // element offset of the tree's current normal-equation block
    int32_t n_chunks;    // sample chunks (work items) per evaluation
    uint16_t n_spill;    // spill slots used
    uint8_t  n_tape;     // tape slots used
    uint8_t  flags;      // TD_UNIQUE_CONST: every rank 0..K-1 occurs exactly once
};
static_assert(sizeof(TreeDesc) == 48, "TreeDesc layout");
constexpr uint8_t TD_UNIQUE_CONST = 1;

// Sizes of the normal-equation block of a tree with K constants:
//   [0, K(K+1)/2)      JtJ lower triangle, row-major packed (i*(i+1)/2 + j, j <= i)
//   [.., + K)          Jtr
//   [.., + 1)          0.5 * sum r^2
__host__ __device__ constexpr inline int nblock_size(int K) { return K * (K + 1) / 2 + K + 1; }

}  // namespace cusr
