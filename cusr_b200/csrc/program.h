// program.h — the compiled tree program executed by the device interpreter.
//
// The pop.bin bytecode (prefix order, one node per slot: nt/nv/ci, cusr/kernel/pop_format.h)
// is compiled on the host, once per call, into two short register-stack programs:
//
//   forward  — evaluates the tree: the value being built lives in a register ("TOS") of every
//              thread; VAR and CONST leaves that feed a binary operator are folded into it as
//              its source operand; two non-leaf children are evaluated in Sethi–Ullman order
//              (the one that needs more stack first) so the shared-memory spill stack is as
//              shallow as it can be; the order of evaluation changes no value (every node
//              still computes `left OP right` of the same operands,
//              cusr/kernel/lm_core.cuh:85-101). Instructions that have a reverse-mode partial
//              write it to their tape slots.
//   reverse  — the adjoint sweep, in reverse order, with the instructions that have no reverse
//              work left out (`+ x`, a leaf load that starts a chain) and every other one
//              reduced to one of a few specialised adjoint updates.
//   row table — after the reverse program, K + 1 bytes packed four to a word: the tape slot
//              holding gradient row k (df/dc_k over the thread's samples), then the slot that
//              takes the residual row. Gradient rows live in tape slots the reverse program
//              has already read for the last time (place_rows in pack.cpp), so they need no
//              storage of their own.
//
// Every opcode is specialised by operator, operand source and operand order, so the
// interpreter's cases are straight-line code.
//
// Word (32 bits, both programs):
//   [0,8)   opcode    forward: XOP (xop_*), reverse: BOP (B_*)
//   [8,16)  idx       variable index or constant rank
//   [16,24) sd        spill slot
//   [24,32) ts        first tape slot
// A reverse instruction that writes a gradient row keeps the constant's rank in `idx` and
// names the row's tape slot in `sd` (in `ts` for B_GRAD_RESTORE, whose `sd` is the spill slot
// it restores from); with the B_ACC bit in its opcode byte (a separate opcode of the
// interpreter) it adds to the row instead of storing it (second and later occurrences of a
// constant).
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

__host__ __device__ constexpr inline uint32_t enc(uint32_t code, uint32_t idx, uint32_t sd,
                                                  uint32_t ts) {
    return (code & 255u) | ((idx & 255u) << 8) | ((sd & 255u) << 16) | ((ts & 255u) << 24);
}
__host__ __device__ inline uint32_t w_code(uint32_t w) { return w & 255u; }
__host__ __device__ inline uint32_t w_idx(uint32_t w)  { return (w >> 8) & 255u; }
__host__ __device__ inline uint32_t w_sd(uint32_t w)   { return (w >> 16) & 255u; }
__host__ __device__ inline uint32_t w_ts(uint32_t w)   { return (w >> 24) & 255u; }

// forward opcodes
constexpr uint32_t XOP_LOAD_VAR = 0, XOP_LOAD_CONST = 1, XOP_PUSH_VAR = 2, XOP_PUSH_CONST = 3;
// unary operator u (OP_SIN .. OP_UZERO)
__host__ __device__ constexpr inline uint32_t xop_un(uint32_t op) { return 8u + (op - OP_SIN); }
// binary operator (OP_ADD .. OP_BZERO) with source mode (M_VAR / M_CONST / M_POP) and order
__host__ __device__ constexpr inline uint32_t xop_bin(uint32_t op, uint32_t mode, uint32_t swap) {
    return 32u + (op - OP_ADD) * 6u + (mode == M_VAR ? 0u : (mode == M_CONST ? 2u : 4u)) + swap;
}

// reverse opcodes (t0 = tape[ts], t1 = tape[ts+1], safe = exact-zero annihilating product)
enum BOp : uint32_t {
    B_GRAD = 0,          // grad[idx] <- adj
    B_GRAD_RESTORE,      // grad[idx] <- adj; adj <- spill[sd]
    B_RESTORE,           // adj <- spill[sd]
    B_GRAD_NEG,          // grad[idx] <- -adj
    B_SPILL,             // spill[sd] <- adj
    B_SPILL_NEG,         // spill[sd] <- -adj
    B_NEG,               // adj <- -adj
    B_GRAD_THEN_NEG,     // grad[idx] <- adj; adj <- -adj
    B_SPILL_THEN_NEG,    // spill[sd] <- adj; adj <- -adj
    B_SCALE_X,           // adj <- safe(adj, x[idx])
    B_SCALE_T0,          // adj <- safe(adj, t0)
    B_MULC,              // grad[idx] <- safe(adj, t0); adj <- safe(adj, c[idx])
    B_GRAD_T1_T0,        // grad[idx] <- safe(adj, t1); adj <- safe(adj, t0)
    B_SPILL_T1_T0,       // spill[sd] <- safe(adj, t1); adj <- safe(adj, t0)
    B_GRAD_1MT0_T0,      // grad[idx] <- safe(adj, 1 - t0); adj <- safe(adj, t0)
    B_SPILL_1MT0_T0,     // spill[sd] <- safe(adj, 1 - t0); adj <- safe(adj, t0)
    B_ZERO,              // adj <- 0
    B_GRAD_ZERO,         // grad[idx] <- 0; adj <- 0
    B_SPILL_ZERO,        // spill[sd] <- 0; adj <- 0
    B_SCALE_1MT0,        // adj <- safe(adj, 1 - t0)
    B_SCALE2_T,          // adj <- safe(safe(adj, t0), tape[idx])   (two chained unary nodes)
    B_ROW_ZERO,          // tape[ts] <- 0   (the shared row of constants absent from the tree)
    B_COUNT
};
// "grad[k]" above is the gradient row of constant k, held in the tape slot the word names
constexpr uint32_t B_ACC = 32u;       // opcode-byte flag of a row write: add instead of store
__host__ __device__ inline uint32_t w_bop(uint32_t w) { return w & 31u; }
// the field of a row-writing word that names the row's tape slot
__host__ __device__ inline uint32_t w_row(uint32_t w) {
    return (w & 31u) == B_GRAD_RESTORE ? w_ts(w) : w_sd(w);
}
__host__ __device__ inline bool is_row_write(uint32_t b) {
    return b == B_GRAD || b == B_GRAD_RESTORE || b == B_GRAD_NEG || b == B_GRAD_THEN_NEG ||
           b == B_MULC || b == B_GRAD_T1_T0 || b == B_GRAD_1MT0_T0 || b == B_GRAD_ZERO;
}
// 32-bit words of the row table of a tree with K constants (K + 1 bytes)
__host__ __device__ constexpr inline int row_table_words(int K) { return (K + 4) / 4; }

constexpr int PROG_MAX_SPILL = 63;   // spill slots
constexpr int PROG_MAX_TAPE  = 255;  // ts field (+1 for two-slot entries)

// The opcodes the device interpreter has a case for (its switch has no bounds check).
__host__ __device__ inline bool valid_forward_code(uint32_t c) {
    if (c <= XOP_PUSH_CONST) return true;
    if (c >= xop_un(OP_SIN) && c <= xop_un(OP_UZERO)) return true;
    if (c < 32u || c > xop_bin(OP_BZERO, M_POP, 1)) return false;
    const uint32_t op = OP_ADD + (c - 32u) / 6u, swap = (c - 32u) & 1u;
    const bool unordered = op == OP_ADD || op == OP_MUL || op == OP_LT || op == OP_GT ||
                           op == OP_LE || op == OP_GE || op == OP_BZERO;
    return !(unordered && swap);
}
__host__ __device__ inline bool valid_reverse_code(uint32_t c) {
    if (c & ~63u) return false;
    if ((c & 31u) >= B_COUNT) return false;
    return !(c & B_ACC) || is_row_write(c & 31u);
}

// Per-tree descriptor uploaded to the device (64 bytes).
struct TreeDesc {
    int32_t code_off;    // first forward instruction in the code array
    int32_t n_instr;     // forward instructions
    int32_t bcode_off;   // first reverse instruction
    int32_t n_bwd;       // reverse instructions
    int32_t K;           // constants of the tree
    int32_t c_off;       // offset of the tree's constants
    int64_t y_off;       // element offset of the tree's target row (0 when shared)
    int64_t p_off;       // element offset of the tree's per-chunk partial sums
    int64_t q_off;       // element offset of the tree's current normal-equation block
    int32_t n_chunks;    // sample chunks (work items) per evaluation
    uint16_t n_spill;    // spill slots used
    uint8_t  n_tape;     // tape slots used
    uint8_t  flags;      // TD_UNIQUE_CONST: every rank 0..K-1 occurs exactly once
    int32_t pad[2];
};
static_assert(sizeof(TreeDesc) == 64, "TreeDesc layout");
constexpr uint8_t TD_UNIQUE_CONST = 1;

// Sizes of the normal-equation block of a tree with K constants:
//   [0, K(K+1)/2)      JtJ lower triangle, row-major packed (i*(i+1)/2 + j, j <= i)
//   [.., + K)          Jtr
//   [.., + 1)          0.5 * sum r^2
__host__ __device__ constexpr inline int nblock_size(int K) { return K * (K + 1) / 2 + K + 1; }

}  // namespace cusr
