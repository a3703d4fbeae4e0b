// eval_kernel.cuh — the fused per-iteration pass of the batched LM engine.
//
// One launch evaluates, for every (tree, sample-chunk) work item of one scheduler bin:
//   value f(x_i; c) of the tree at every sample        (cusr/kernel/lm_core.cuh:58-125)
//   its gradient g_i = df/dc by a reverse sweep         (cusr/kernel/revad_interp.cuh:66-191)
//   the residual r_i = f - y_i and, summed over the chunk,
//   JtJ (lower triangle), Jtr and sum r^2               (lm_core.cuh:127-177)
// and writes those sums to a per-item slot; the LM step kernel adds the slots of a tree in
// a fixed order, so results do not depend on which block ran which item.
//
// The reference runs this as five kernels with the Jacobian materialised in HBM
// (d_J[M*K_max*N], co_lib.cu:233, 351, 388); here J rows never leave the SM.
//
// Execution model (B200 / sm_100a):
//   * persistent blocks of NT threads pull work items from an atomic counter; items of a
//     bin are ordered most-expensive-tree first (LPT);
//   * every thread evaluates V consecutive samples at once (instruction decode is amortised
//     over V samples and the V chains give independent instructions);
//   * the forward and reverse programs (program.h; warp-uniform, every opcode specialised so
//     each case is straight-line code) and the constants sit in shared memory; each thread's
//     spill stack, reverse tape and input row are private shared-memory columns laid out
//     [slot][thread] (conflict-free, no block barriers inside an item);
//   * the gradient rows (df/dc_k over the thread's samples) and the residual row are written
//     into tape slots the reverse program no longer needs (the compiler's row table names
//     them), so they take no shared memory of their own (a launch whose tape is in global
//     memory keeps them in a small shared-memory row region instead);
//   * each warp forms the (K+1)x(K+1) Gram matrix of [g; r] over its samples on the fp64
//     tensor cores, straight from those rows; its packed lower triangle is the partial layout
//     (JtJ, Jtr, sum r^2). KC = constant-count class of the bin (K <= KC); KC = 1, 2 run the
//     forward-mode tangent sweep instead, with the sums in registers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/cusr_co.h"
#include "program.h"
#include "ops.h"

namespace cusr {

template <typename T, int V> struct alignas(sizeof(T) * V) VecT { T v[V]; };
template <int V> struct alignas(4 * V) VecF { float v[V]; };

template <typename T>
struct EvalParams {
    const uint32_t *code;
    const TreeDesc *desc;
    const int2 *items;       // {tree, chunk}
    const int *n_items;      // number of items of this launch (device)
    int *counter;            // work counter (reset to 0 by the item builder)
    const T *c;              // constants of the evaluated point, indexed by TreeDesc::c_off
    const float *xs;         // inputs, [n_vars][ldx]
    const float *ym;         // targets, row of tree m at TreeDesc::y_off
    T *partials;             // per-item sums, slot TreeDesc::p_off + chunk * nblock_size(K)
    int64_t ldx;
    int N;
    int chunk;               // samples per item (multiple of NT * V)
    int n_vars;
    int code_cap;            // shared-memory words reserved for the two programs of a tree
    int spill_cap;           // spill slots reserved per thread
    int tape_cap;            // tape slots reserved per thread
    void *tape_g;            // global tape (TG instantiations): [block][tape_cap][thread]
    T *vals;                 // optional: per-sample values, [tree][N]
    T *jac;                  // optional: per-sample gradients, [tree][jac_kmax][N]
    int jac_kmax;
    // optional per-fit mode bits (indexed like desc); IM_SENTINEL fits take the residual
    // convention of the reference's scipy backend
    const uint8_t *imode = nullptr;
};

// Per-fit mode bit: a non-finite residual counts as the sentinel 1e6 with a zero gradient
// row, the objective the reference's scipy backend hands to MINPACK
// (cusr/benchmark/backends.py:105-110: np.where(np.isfinite(r), r, 1e6); a forward
// difference across two sentinel values is 0). Set for the trust-region fits.
constexpr uint8_t IM_SENTINEL = 4;
constexpr double RESIDUAL_SENTINEL = 1e6;

__host__ __device__ constexpr inline size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

// Shared-memory layout of one block; the host sizes the launch with the same function.
// KC = 1, 2: forward-mode classes (tangents in registers, no tape, no gradient rows; a spill
// slot holds the value and its KC tangents).
// KC >= 4: reverse mode; a tape slot is NT VecT entries plus a pad of 4 elements of T, so
// that a slot used as a gradient row starts 4 banks (fp32) further on than the slot before:
// the eight rows of a tensor-core fragment load land in distinct banks when the compiler
// gives them distinct slot residues mod 8. When the tape lives in global memory (trees too
// long for shared memory), the KC + 1 gradient and residual rows get a shared-memory region
// of their own, row k for constant k and row K for the residual.
template <typename T, int V, int NT, int KC>
struct EvalSmem {
    static constexpr bool kFwd = KC <= 2;
    static constexpr int kTapeStride = NT + 4 / V;            // VecT entries per tape slot
    static constexpr int kSpillWords = kFwd ? 1 + KC : 1;     // VecT entries per spill slot
    size_t code, cval, x, spill, tape, rows, red, total;
    __host__ __device__ EvalSmem(int code_cap, int n_vars, int spill_cap, int tape_cap,
                                 bool tape_in_smem = true) {
        size_t o = 0;
        code = o;  o += align16((size_t)(code_cap + 1) * 4);
        cval = o;  o += align16((size_t)CO_MAX_K * sizeof(T));
        x = o;     o += align16((size_t)n_vars * NT * V * 4);
        spill = o; o += align16((size_t)spill_cap * kSpillWords * NT * V * sizeof(T));
        tape = o;
        o += (tape_in_smem && !kFwd) ? align16((size_t)tape_cap * kTapeStride * V * sizeof(T)) : 0;
        rows = o;
        o += (!tape_in_smem && !kFwd) ? align16((size_t)(KC + 1) * kTapeStride * V * sizeof(T)) : 0;
        red = o;   o += align16((size_t)(NT / 32) * nblock_size(KC) * sizeof(T));
        total = o;
    }
};

#define CUSR_FOR_V _Pragma("unroll") for (int j = 0; j < V; ++j)

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T, int V>
__device__ __forceinline__ VecT<T, V> pack(const T (&a)[V]) {
    VecT<T, V> r;
    CUSR_FOR_V r.v[j] = a[j];
    return r;
}

// ---------------------------------------------------------------------------------------
// Forward sweep. xt / sp / tp point at this thread's column (x_s + tid, ...); slot k of a
// column is element k * NT.
// ---------------------------------------------------------------------------------------
template <typename T, int V, int NT, int TSTR, bool GRAD, uint32_t OP, uint32_t MODE, bool SW>
__device__ __forceinline__ void fwd_bin(uint32_t w, const T *__restrict__ c_s,
                                        const VecF<V> *__restrict__ xt,
                                        const VecT<T, V> *__restrict__ sp,
                                        VecT<T, V> *__restrict__ tp, T (&tos)[V]) {
    T s[V];
    if constexpr (MODE == M_VAR) {
        const VecF<V> xv = xt[w_idx(w) * NT];
        CUSR_FOR_V s[j] = (T)xv.v[j];
    } else if constexpr (MODE == M_CONST) {
        const T cv = c_s[w_idx(w)];
        CUSR_FOR_V s[j] = cv;
    } else {
        const VecT<T, V> t = sp[w_sd(w) * NT];
        CUSR_FOR_V s[j] = t.v[j];
    }
    T o[V], dt[V], ds[V];
    CUSR_FOR_V {
        T da, db;
        binary_op<T>(OP, SW ? s[j] : tos[j], SW ? tos[j] : s[j], o[j], da, db);
        dt[j] = SW ? db : da;
        ds[j] = SW ? da : db;
    }
    if constexpr (GRAD) {
        const int ts = (int)w_ts(w);
        if constexpr (OP == OP_MUL) {
            if constexpr (MODE == M_CONST) {
                tp[ts * TSTR] = pack<T, V>(ds);
            } else if constexpr (MODE == M_POP) {
                tp[ts * TSTR] = pack<T, V>(dt);
                tp[(ts + 1) * TSTR] = pack<T, V>(ds);
            }
        } else if constexpr (OP == OP_DIV || OP == OP_POW || OP == OP_POWABS) {
            tp[ts * TSTR] = pack<T, V>(dt);
            if constexpr (MODE != M_VAR) tp[(ts + 1) * TSTR] = pack<T, V>(ds);
        } else if constexpr (OP == OP_MAX || OP == OP_MIN) {
            tp[ts * TSTR] = pack<T, V>(dt);
        }
    }
    CUSR_FOR_V tos[j] = o[j];
}

template <typename T, int V, int TSTR, bool GRAD, uint32_t OP>
__device__ __forceinline__ void fwd_un(uint32_t w, VecT<T, V> *__restrict__ tp, T (&tos)[V]) {
    T d[V];
    CUSR_FOR_V {
        T r;
        unary_op<T>(OP, tos[j], r, d[j]);
        tos[j] = r;
    }
    if constexpr (GRAD && OP != OP_NEG && OP != OP_UZERO) tp[w_ts(w) * TSTR] = pack<T, V>(d);
}

// TSTR: VecT entries between consecutive tape slots
template <typename T, int V, int NT, int TSTR, bool GRAD>
__device__ __forceinline__ void forward_sweep(const uint32_t *__restrict__ code, int n,
                                              const T *__restrict__ c_s,
                                              const VecF<V> *__restrict__ xt,
                                              VecT<T, V> *__restrict__ sp,
                                              VecT<T, V> *__restrict__ tp, T (&tos)[V]) {
    uint32_t wn = code[0];
    for (int pc = 0; pc < n; ++pc) {
        const uint32_t w = wn;
        wn = code[pc + 1];   // next word in flight while this one executes (programs are padded)
        switch (w_code(w)) {
            case XOP_PUSH_VAR:
                sp[w_sd(w) * NT] = pack<T, V>(tos);
                [[fallthrough]];
            case XOP_LOAD_VAR: {
                const VecF<V> xv = xt[w_idx(w) * NT];
                CUSR_FOR_V tos[j] = (T)xv.v[j];
                break;
            }
            case XOP_PUSH_CONST:
                sp[w_sd(w) * NT] = pack<T, V>(tos);
                [[fallthrough]];
            case XOP_LOAD_CONST: {
                const T cv = c_s[w_idx(w)];
                CUSR_FOR_V tos[j] = cv;
                break;
            }
#define CUSR_UN(OPC) case xop_un(OPC): fwd_un<T, V, TSTR, GRAD, OPC>(w, tp, tos); break;
            CUSR_UN(OP_SIN) CUSR_UN(OP_COS) CUSR_UN(OP_LOG) CUSR_UN(OP_LOGABS)
            CUSR_UN(OP_SQRT) CUSR_UN(OP_SQRTABS)
            CUSR_UN(OP_TAN) CUSR_UN(OP_SINH) CUSR_UN(OP_COSH) CUSR_UN(OP_TANH)
            CUSR_UN(OP_EXP) CUSR_UN(OP_INV) CUSR_UN(OP_NEG) CUSR_UN(OP_ABS) CUSR_UN(OP_UZERO)
#undef CUSR_UN
#define CUSR_B(OPC, MODE, SW)                                                          \
    case xop_bin(OPC, MODE, SW):                                                       \
        fwd_bin<T, V, NT, TSTR, GRAD, OPC, MODE, SW>(w, c_s, xt, sp, tp, tos);         \
        break;
// operand order matters: every (mode, order); commutative ones are emitted unswapped
#define CUSR_B6(OPC) CUSR_B(OPC, M_VAR, 0) CUSR_B(OPC, M_VAR, 1) CUSR_B(OPC, M_CONST, 0) \
                     CUSR_B(OPC, M_CONST, 1) CUSR_B(OPC, M_POP, 0) CUSR_B(OPC, M_POP, 1)
#define CUSR_B3(OPC) CUSR_B(OPC, M_VAR, 0) CUSR_B(OPC, M_CONST, 0) CUSR_B(OPC, M_POP, 0)
            CUSR_B3(OP_ADD) CUSR_B6(OP_SUB) CUSR_B3(OP_MUL) CUSR_B6(OP_DIV)
            CUSR_B6(OP_POW) CUSR_B6(OP_POWABS) CUSR_B6(OP_MAX) CUSR_B6(OP_MIN)
            CUSR_B3(OP_LT) CUSR_B3(OP_GT) CUSR_B3(OP_LE) CUSR_B3(OP_GE) CUSR_B3(OP_BZERO)
#undef CUSR_B3
#undef CUSR_B6
#undef CUSR_B
            default:
                // every word was checked against this case set on the host
                // (valid_forward_code / valid_reverse_code), so no bounds check is needed
                __builtin_unreachable();
        }
    }
}

// ---------------------------------------------------------------------------------------
// Forward-mode sweep (KC = KT <= 2): the same forward program; TOS carries its value and the
// KT tangents d/dc_k. A VAR leaf has tangent 0, CONST leaf k the unit vector e_k; an operator
// maps tangents by its local partials with the reverse sweep's zero-annihilating product
// (t <- safe(d, t); a binary node adds the source operand's term). The result equals the
// reverse sweep's product of partials along each root-to-leaf path, taken leaf to root.
// ---------------------------------------------------------------------------------------
template <typename T, int V, int NT, int KT>
__device__ __forceinline__ void tan_push(VecT<T, V> *__restrict__ sp, uint32_t sd,
                                         const T (&tos)[V], const T (&tt)[KT][V]) {
    VecT<T, V> *s = sp + (int)sd * (1 + KT) * NT;
    s[0] = pack<T, V>(tos);
#pragma unroll
    for (int k = 0; k < KT; ++k) s[(1 + k) * NT] = pack<T, V>(tt[k]);
}

template <typename T, int V, int NT, int KT, uint32_t OP, uint32_t MODE, bool SW>
__device__ __forceinline__ void tan_bin(uint32_t w, const T *__restrict__ c_s,
                                        const VecF<V> *__restrict__ xt,
                                        const VecT<T, V> *__restrict__ sp, T (&tos)[V],
                                        T (&tt)[KT][V]) {
    T s[V];
    T ts[KT][V];
    if constexpr (MODE == M_VAR) {
        const VecF<V> xv = xt[w_idx(w) * NT];
        CUSR_FOR_V s[j] = (T)xv.v[j];
    } else if constexpr (MODE == M_CONST) {
        const T cv = c_s[w_idx(w)];
        CUSR_FOR_V s[j] = cv;
    } else {
        const VecT<T, V> *q = sp + (int)w_sd(w) * (1 + KT) * NT;
        const VecT<T, V> t = q[0];
        CUSR_FOR_V s[j] = t.v[j];
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            const VecT<T, V> u = q[(1 + k) * NT];
            CUSR_FOR_V ts[k][j] = u.v[j];
        }
    }
    CUSR_FOR_V {
        T o, da, db;
        binary_op<T>(OP, SW ? s[j] : tos[j], SW ? tos[j] : s[j], o, da, db);
        const T dt = SW ? db : da, ds = SW ? da : db;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            T t = safe_mul(dt, tt[k][j]);
            if constexpr (MODE == M_CONST) {
                if ((uint32_t)k == w_idx(w)) t += ds;
            } else if constexpr (MODE == M_POP) {
                t += safe_mul(ds, ts[k][j]);
            }
            tt[k][j] = t;
        }
        tos[j] = o;
    }
}

template <typename T, int V, int NT, int KT, uint32_t OP>
__device__ __forceinline__ void tan_un(T (&tos)[V], T (&tt)[KT][V]) {
    CUSR_FOR_V {
        T r, d;
        unary_op<T>(OP, tos[j], r, d);
        tos[j] = r;
#pragma unroll
        for (int k = 0; k < KT; ++k) tt[k][j] = safe_mul(d, tt[k][j]);
    }
}

template <typename T, int V, int NT, int KT>
__device__ __forceinline__ void tangent_sweep(const uint32_t *__restrict__ code, int n,
                                              const T *__restrict__ c_s,
                                              const VecF<V> *__restrict__ xt,
                                              VecT<T, V> *__restrict__ sp, T (&tos)[V],
                                              T (&tt)[KT][V]) {
    uint32_t wn = code[0];
    for (int pc = 0; pc < n; ++pc) {
        const uint32_t w = wn;
        wn = code[pc + 1];
        switch (w_code(w)) {
            case XOP_PUSH_VAR:
                tan_push<T, V, NT, KT>(sp, w_sd(w), tos, tt);
                [[fallthrough]];
            case XOP_LOAD_VAR: {
                const VecF<V> xv = xt[w_idx(w) * NT];
                CUSR_FOR_V {
                    tos[j] = (T)xv.v[j];
#pragma unroll
                    for (int k = 0; k < KT; ++k) tt[k][j] = T(0);
                }
                break;
            }
            case XOP_PUSH_CONST:
                tan_push<T, V, NT, KT>(sp, w_sd(w), tos, tt);
                [[fallthrough]];
            case XOP_LOAD_CONST: {
                const uint32_t idx = w_idx(w);
                const T cv = c_s[idx];
                CUSR_FOR_V {
                    tos[j] = cv;
#pragma unroll
                    for (int k = 0; k < KT; ++k) tt[k][j] = (uint32_t)k == idx ? T(1) : T(0);
                }
                break;
            }
#define CUSR_UN(OPC) case xop_un(OPC): tan_un<T, V, NT, KT, OPC>(tos, tt); break;
            CUSR_UN(OP_SIN) CUSR_UN(OP_COS) CUSR_UN(OP_TAN) CUSR_UN(OP_SINH)
            CUSR_UN(OP_COSH) CUSR_UN(OP_TANH) CUSR_UN(OP_LOG) CUSR_UN(OP_LOGABS)
            CUSR_UN(OP_EXP) CUSR_UN(OP_INV) CUSR_UN(OP_NEG) CUSR_UN(OP_ABS)
            CUSR_UN(OP_SQRT) CUSR_UN(OP_SQRTABS) CUSR_UN(OP_UZERO)
#undef CUSR_UN
#define CUSR_B(OPC, MODE, SW)                                                          \
    case xop_bin(OPC, MODE, SW):                                                       \
        tan_bin<T, V, NT, KT, OPC, MODE, SW>(w, c_s, xt, sp, tos, tt);                 \
        break;
#define CUSR_B6(OPC) CUSR_B(OPC, M_VAR, 0) CUSR_B(OPC, M_VAR, 1) CUSR_B(OPC, M_CONST, 0) \
                     CUSR_B(OPC, M_CONST, 1) CUSR_B(OPC, M_POP, 0) CUSR_B(OPC, M_POP, 1)
#define CUSR_B3(OPC) CUSR_B(OPC, M_VAR, 0) CUSR_B(OPC, M_CONST, 0) CUSR_B(OPC, M_POP, 0)
            CUSR_B3(OP_ADD) CUSR_B6(OP_SUB) CUSR_B3(OP_MUL) CUSR_B6(OP_DIV)
            CUSR_B6(OP_POW) CUSR_B6(OP_POWABS) CUSR_B6(OP_MAX) CUSR_B6(OP_MIN)
            CUSR_B3(OP_LT) CUSR_B3(OP_GT) CUSR_B3(OP_LE) CUSR_B3(OP_GE) CUSR_B3(OP_BZERO)
#undef CUSR_B3
#undef CUSR_B6
#undef CUSR_B
            default:
                __builtin_unreachable();   // host-validated opcodes
        }
    }
}

// Where a thread's gradient rows are: in its tape column, at the row slots the compiler chose
// (ROWS = false), or, for a global tape, in its column of the shared-memory row region, row k
// for constant k (ROWS = true). RS = VecT entries between rows.
template <typename T, int V, int RS, bool ROWS>
struct RowCol {
    VecT<T, V> *rp;
    __device__ __forceinline__ VecT<T, V> *at(uint32_t k, uint32_t slot) const {
        return rp + (int)(ROWS ? k : slot) * RS;
    }
};

// gradient row write of word w: this thread's entry of the row, stored, or added to for the
// second and later occurrences of a constant (the B_ACC opcodes)
template <uint32_t B, typename T, int V, int RS, bool ROWS, bool ACC>
__device__ __forceinline__ void row_put(const RowCol<T, V, RS, ROWS> &rc, uint32_t w,
                                        const T (&a)[V]) {
    // the slot field of opcode B (w_row, resolved at compile time)
    VecT<T, V> *q = rc.at(w_idx(w), B == B_GRAD_RESTORE ? w_ts(w) : w_sd(w));
    if constexpr (ACC) {
        VecT<T, V> o = *q;
        CUSR_FOR_V o.v[j] += a[j];
        *q = o;
    } else {
        *q = pack<T, V>(a);
    }
}

// ---------------------------------------------------------------------------------------
// Reverse sweep over the reverse program: adjoints from the root to the leaves; the gradient
// row of constant k (df/dc_k) is written to the row slot the instruction names. Every
// (opcode, store / add) pair is its own case of the dispatch, so each is straight-line code.
// ---------------------------------------------------------------------------------------
template <uint32_t B, bool ACC, typename T, int V, int NT, int TSTR, int RS, bool ROWS>
__device__ __forceinline__ void rev_step(uint32_t w, T (&adj)[V], const T *__restrict__ c_s,
                                         const VecF<V> *__restrict__ xt,
                                         VecT<T, V> *__restrict__ sp, VecT<T, V> *tp,
                                         const RowCol<T, V, RS, ROWS> &rc) {
    typedef VecT<T, V> VT;
    if constexpr (B == B_GRAD) {
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, adj);
    } else if constexpr (B == B_GRAD_RESTORE) {
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, adj);
        const VT t = sp[w_sd(w) * NT];
        CUSR_FOR_V adj[j] = t.v[j];
    } else if constexpr (B == B_RESTORE) {
        const VT t = sp[w_sd(w) * NT];
        CUSR_FOR_V adj[j] = t.v[j];
    } else if constexpr (B == B_GRAD_NEG) {
        T a[V];
        CUSR_FOR_V a[j] = -adj[j];
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, a);
    } else if constexpr (B == B_SPILL) {
        sp[w_sd(w) * NT] = pack<T, V>(adj);
    } else if constexpr (B == B_SPILL_NEG) {
        T a[V];
        CUSR_FOR_V a[j] = -adj[j];
        sp[w_sd(w) * NT] = pack<T, V>(a);
    } else if constexpr (B == B_NEG) {
        CUSR_FOR_V adj[j] = -adj[j];
    } else if constexpr (B == B_GRAD_THEN_NEG) {
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, adj);
        CUSR_FOR_V adj[j] = -adj[j];
    } else if constexpr (B == B_SPILL_THEN_NEG) {
        sp[w_sd(w) * NT] = pack<T, V>(adj);
        CUSR_FOR_V adj[j] = -adj[j];
    } else if constexpr (B == B_SCALE_X) {
        const VecF<V> xv = xt[w_idx(w) * NT];
        CUSR_FOR_V adj[j] = safe_mul(adj[j], (T)xv.v[j]);
    } else if constexpr (B == B_SCALE_T0) {
        const VT t0 = tp[w_ts(w) * TSTR];
        CUSR_FOR_V adj[j] = safe_mul(adj[j], t0.v[j]);
    } else if constexpr (B == B_MULC) {
        const VT t0 = tp[w_ts(w) * TSTR];
        const T cv = c_s[w_idx(w)];
        T a[V];
        CUSR_FOR_V { a[j] = safe_mul(adj[j], t0.v[j]); adj[j] = safe_mul(adj[j], cv); }
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, a);
    } else if constexpr (B == B_GRAD_T1_T0 || B == B_SPILL_T1_T0) {
        const int ts = (int)w_ts(w);
        const VT t0 = tp[ts * TSTR], t1 = tp[(ts + 1) * TSTR];
        T a[V];
        CUSR_FOR_V { a[j] = safe_mul(adj[j], t1.v[j]); adj[j] = safe_mul(adj[j], t0.v[j]); }
        if constexpr (B == B_GRAD_T1_T0) row_put<B, T, V, RS, ROWS, ACC>(rc, w, a);
        else sp[w_sd(w) * NT] = pack<T, V>(a);
    } else if constexpr (B == B_GRAD_1MT0_T0 || B == B_SPILL_1MT0_T0) {
        const VT t0 = tp[w_ts(w) * TSTR];
        T a[V];
        CUSR_FOR_V { a[j] = safe_mul(adj[j], T(1) - t0.v[j]); adj[j] = safe_mul(adj[j], t0.v[j]); }
        if constexpr (B == B_GRAD_1MT0_T0) row_put<B, T, V, RS, ROWS, ACC>(rc, w, a);
        else sp[w_sd(w) * NT] = pack<T, V>(a);
    } else if constexpr (B == B_ZERO) {
        CUSR_FOR_V adj[j] = T(0);
    } else if constexpr (B == B_GRAD_ZERO) {
        T a[V];
        CUSR_FOR_V { a[j] = T(0); adj[j] = T(0); }
        row_put<B, T, V, RS, ROWS, ACC>(rc, w, a);
    } else if constexpr (B == B_SPILL_ZERO) {
        T a[V];
        CUSR_FOR_V { a[j] = T(0); adj[j] = T(0); }
        sp[w_sd(w) * NT] = pack<T, V>(a);
    } else if constexpr (B == B_SCALE2_T) {
        const VT t0 = tp[w_ts(w) * TSTR], t1 = tp[w_idx(w) * TSTR];
        CUSR_FOR_V adj[j] = safe_mul(safe_mul(adj[j], t0.v[j]), t1.v[j]);
    } else if constexpr (B == B_SCALE_1MT0) {
        const VT t0 = tp[w_ts(w) * TSTR];
        CUSR_FOR_V adj[j] = safe_mul(adj[j], T(1) - t0.v[j]);
    } else if constexpr (B == B_ROW_ZERO) {
        // the shared zero row of absent constants (a row region is zeroed per tree instead)
        if constexpr (!ROWS) {
            T a[V];
            CUSR_FOR_V a[j] = T(0);
            tp[w_ts(w) * TSTR] = pack<T, V>(a);
        }
    }
}

template <typename T, int V, int NT, int TSTR, int RS, bool ROWS>
__device__ __forceinline__ void reverse_sweep(const uint32_t *__restrict__ code, int n,
                                              const T *__restrict__ c_s,
                                              const VecF<V> *__restrict__ xt,
                                              VecT<T, V> *__restrict__ sp, VecT<T, V> *tp,
                                              const RowCol<T, V, RS, ROWS> rc) {
    T adj[V];
    CUSR_FOR_V adj[j] = T(1);
    uint32_t wn = code[0];
    for (int pc = 0; pc < n; ++pc) {
        const uint32_t w = wn;
        wn = code[pc + 1];
        switch (w_code(w)) {
#define CUSR_R(B) case B: rev_step<B, false, T, V, NT, TSTR, RS, ROWS>(w, adj, c_s, xt, sp, tp, rc); break;
#define CUSR_RA(B) CUSR_R(B) \
    case B | B_ACC: rev_step<B, true, T, V, NT, TSTR, RS, ROWS>(w, adj, c_s, xt, sp, tp, rc); break;
            CUSR_RA(B_GRAD) CUSR_RA(B_GRAD_RESTORE) CUSR_R(B_RESTORE) CUSR_RA(B_GRAD_NEG)
            CUSR_R(B_SPILL) CUSR_R(B_SPILL_NEG) CUSR_R(B_NEG) CUSR_RA(B_GRAD_THEN_NEG)
            CUSR_R(B_SPILL_THEN_NEG) CUSR_R(B_SCALE_X) CUSR_R(B_SCALE_T0) CUSR_RA(B_MULC)
            CUSR_RA(B_GRAD_T1_T0) CUSR_R(B_SPILL_T1_T0) CUSR_RA(B_GRAD_1MT0_T0)
            CUSR_R(B_SPILL_1MT0_T0) CUSR_R(B_ZERO) CUSR_RA(B_GRAD_ZERO) CUSR_R(B_SPILL_ZERO)
            CUSR_R(B_SCALE_1MT0) CUSR_R(B_SCALE2_T) CUSR_R(B_ROW_ZERO)
#undef CUSR_RA
#undef CUSR_R
            default:
                // every word was checked against this case set on the host
                // (valid_forward_code / valid_reverse_code), so no bounds check is needed
                __builtin_unreachable();
        }
    }
}

// D(8x8) += A(8x4) B(4x8) on the fp64 tensor cores (mma.sync m8n8k4 .f64). Fragments: a
// lane holds A[lane / 4][lane % 4], B[lane % 4][lane / 4] and D[lane / 4][2 (lane % 4) + q].
__device__ __forceinline__ void dmma_884(double (&c)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(c[0]), "+d"(c[1])
                 : "d"(a), "d"(b));
}

// ---------------------------------------------------------------------------------------
// The fused evaluation kernel.
//   T     arithmetic type (float / double)
//   V     samples per thread
//   NT    threads per block
//   KC    constant-count class of the bin (trees with K <= KC)
//   GRAD  gradients and normal equations (the engine launches GRAD = true only; value-only
//         passes run lm_value_kernel below); a tree with K = 0 takes the value-and-loss path
//   TG    reverse tape in global scratch instead of shared memory
//   FAST  instantiated in the translation unit built with the reference kernel's
//         --use_fast_math flags (approximate transcendentals, division and square root,
//         denormals flushed); the source is the same, only the name differs
// ---------------------------------------------------------------------------------------
// Register budget: fp32 classes K <= 16 are held to 64 registers per thread (eight 128-thread
// blocks per SM, as many as shared memory allows for the common tape sizes); the K <= 32
// class keeps its 15 accumulator tiles in registers at four blocks; fp64 (twice the shared
// memory per thread) is held to six and two blocks.
#ifndef CUSR_F64_THREADS_PER_SM
// fp64 classes K <= 16: resident threads per SM (768: 85 registers, small spills; 512 removes
// the spills and measured 0.7-4% slower on the parity mode and the physics configuration)
#define CUSR_F64_THREADS_PER_SM 768
#endif
template <typename T, int V, int NT, int KC, bool GRAD, bool TG, bool FAST>
__global__ void __launch_bounds__(
    NT, (sizeof(T) == 4 ? (KC > 16 ? 512 : 1024) : (KC > 16 ? 256 : CUSR_F64_THREADS_PER_SM)) / NT)
lm_eval_kernel(const EvalParams<T> p) {
    typedef EvalSmem<T, V, NT, KC> L;
    constexpr bool FWD = GRAD && L::kFwd;    // forward-mode tangents (KC = 1, 2)
    constexpr bool REV = GRAD && !L::kFwd;   // reverse sweep + tensor-core normal equations
    constexpr int NTL = REV ? (KC + 1 + 7) / 8 : 1;   // 8-row tiles of [g; r]
    constexpr int NTILE = NTL * (NTL + 1) / 2;        // lower-triangle tiles
    // VecT entries per tape slot: padded in shared memory (slots double as gradient rows);
    // a global tape keeps the rows in shared memory and its slots 128-byte aligned
    constexpr int TSTR = TG ? NT : L::kTapeStride;
    constexpr int RSTR = L::kTapeStride;              // VecT entries per gradient row
    constexpr int ROUND = NT * V;
    constexpr int NW = NT / 32;
    constexpr int NTRI = KC * (KC + 1) / 2;

    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_item, s_sent;
    const L lay(p.code_cap, p.n_vars, p.spill_cap, p.tape_cap, !TG);
    uint32_t *code_s = reinterpret_cast<uint32_t *>(smem + lay.code);
    T *c_s = reinterpret_cast<T *>(smem + lay.cval);
    VecF<V> *x_s = reinterpret_cast<VecF<V> *>(smem + lay.x);
    VecT<T, V> *spill_s = reinterpret_cast<VecT<T, V> *>(smem + lay.spill);
    // reverse tape: private shared-memory columns, whose slots the reverse sweep has finished
    // with also take the gradient and residual rows; or (TG, trees whose tape would not fit
    // beside a second resident block) this block's slab of a global scratch buffer, read back
    // by the same thread and served from L1/L2, with the rows in the shared row region
    VecT<T, V> *tape_s =
        TG ? reinterpret_cast<VecT<T, V> *>(p.tape_g) + (int64_t)blockIdx.x * p.tape_cap * TSTR
           : reinterpret_cast<VecT<T, V> *>(smem + lay.tape);
    T *red_s = reinterpret_cast<T *>(smem + lay.red);
    // global tape: the gradient and residual rows live in a shared-memory region of their own
    VecT<T, V> *rows_s = reinterpret_cast<VecT<T, V> *>(smem + lay.rows);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_items = *p.n_items;
    VecF<V> *xt = x_s + tid;
    VecT<T, V> *spt = spill_s + tid;
    VecT<T, V> *tpt = tape_s + tid;
    const RowCol<T, V, RSTR, TG> rc{TG ? rows_s + tid : tpt};
    const T *row_base = reinterpret_cast<const T *>(TG ? rows_s : tape_s);

    for (;;) {
        if (tid == 0) s_item = atomicAdd(p.counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= n_items) break;
        const int2 wi = p.items[it];
        const TreeDesc d = p.desc[wi.x];
        const int K = d.K;
        const bool grad = GRAD && K > 0;
        // the fit's sentinel bit, read back from shared memory where needed (no register is
        // held across the sweeps for it)
        if (tid == 0) s_sent = p.imode ? (p.imode[wi.x] & IM_SENTINEL) : 0;
        // forward program; for reverse mode the reverse program and its row table follow
        const int n_code = REV ? d.n_instr + d.n_bwd + row_table_words(K) : d.n_instr;
        for (int i = tid; i < n_code; i += NT) code_s[i] = p.code[d.code_off + i];
        if (tid == 0) code_s[n_code] = 0u;   // prefetch pad after the last staged word
        for (int i = tid; i < K; i += NT) c_s[i] = p.c[d.c_off + i];
        if constexpr (REV && TG) {
            // rows of constants absent from the tree are never written: zero them once
            VecT<T, V> z;
            CUSR_FOR_V z.v[j] = T(0);
            for (int k = 0; k < K; ++k) rc.at(k, 0)[0] = z;
        }
        __syncthreads();
        const uint32_t *bcode_s = code_s + d.n_instr;
        // tape slot of row r (r < K: gradient of constant r, r = K: residual)
        const uint8_t *rtab = reinterpret_cast<const uint8_t *>(bcode_s + d.n_bwd);

        // forward mode: sums in registers; reverse mode: fp64 tensor-core fragments of the
        // [g; r] Gram matrix, each lane loading the rows 8 t + lane / 4 of the tiles
        T acc[FWD ? NTRI : 1];
        T jtr[FWD ? KC : 1];
        double cm[REV ? NTILE : 1][2];
        int roff[NTL];
#pragma unroll
        for (int t = 0; t < (REV ? NTILE : 1); ++t) cm[t][0] = cm[t][1] = 0.0;
        if constexpr (FWD) {
#pragma unroll
            for (int e = 0; e < NTRI; ++e) acc[e] = T(0);
#pragma unroll
            for (int e = 0; e < KC; ++e) jtr[e] = T(0);
        }
        if constexpr (REV) {
#pragma unroll
            for (int t = 0; t < NTL; ++t) {
                const int row = 8 * t + (lane >> 2);
                roff[t] = !(grad && row <= K) ? -1 : (TG ? row : (int)rtab[row]) * RSTR * V;
            }
        }
        T lsum = T(0);

        const int64_t s0 = (int64_t)wi.y * p.chunk;
        const int64_t s_end = (int64_t)p.N < s0 + p.chunk ? (int64_t)p.N : s0 + p.chunk;
        const float *yrow = p.ym + d.y_off;
        for (int64_t base = s0; base < s_end; base += ROUND) {
            const int64_t si = base + (int64_t)tid * V;
            for (int v = 0; v < p.n_vars; ++v)
                xt[v * NT] = *reinterpret_cast<const VecF<V> *>(p.xs + (int64_t)v * p.ldx + si);
            const VecF<V> yv = *reinterpret_cast<const VecF<V> *>(yrow + si);

            T f[V];
            T tt[FWD ? KC : 1][V];
            if constexpr (FWD) {
                tangent_sweep<T, V, NT, KC>(code_s, d.n_instr, c_s, xt, spt, f, tt);
            } else {
                forward_sweep<T, V, NT, TSTR, GRAD>(code_s, d.n_instr, c_s, xt, spt, tpt, f);
            }
            T r[V];
            bool valid[V];
            CUSR_FOR_V {
                valid[j] = si + j < p.N;
                r[j] = valid[j] ? f[j] - (T)yv.v[j] : T(0);
            }
            // sentinel fits: non-finite residuals become the sentinel, their samples' gradient
            // entries are dropped (bit j of the mask); applied where the gradients are final
            auto sentinel_mask = [&]() -> unsigned {
                unsigned mk = 0u;
                if (s_sent) {
                    CUSR_FOR_V {
                        if (!Mth<T>::finite(r[j])) {
                            r[j] = T(RESIDUAL_SENTINEL);
                            mk |= 1u << j;
                        }
                    }
                }
                return mk;
            };
            if (p.vals) {
                CUSR_FOR_V if (valid[j]) p.vals[(int64_t)wi.x * p.N + si + j] = f[j];
            }
            if constexpr (FWD) {
              const unsigned mk = sentinel_mask();
              CUSR_FOR_V {
                  if ((mk >> j) & 1u) valid[j] = false;
                  lsum += r[j] * r[j];
              }
              if (grad) {
                if (p.jac) {
                    T *jrow = p.jac + (int64_t)wi.x * p.jac_kmax * p.N;
#pragma unroll
                    for (int k = 0; k < KC; ++k)
                        if (k < K) { CUSR_FOR_V if (valid[j]) jrow[(int64_t)k * p.N + si + j] = tt[k][j]; }
                }
                CUSR_FOR_V {
#pragma unroll
                    for (int i = 0; i < KC; ++i) {
                        if (i < K) {
                            const T gi = valid[j] ? tt[i][j] : T(0);
                            jtr[i] += gi * r[j];
#pragma unroll
                            for (int l = 0; l <= i; ++l)
                                acc[i * (i + 1) / 2 + l] += gi * (valid[j] ? tt[l][j] : T(0));
                        }
                    }
                }
              }
            } else if (!grad) {
                sentinel_mask();
                CUSR_FOR_V lsum += r[j] * r[j];
            } else {
                reverse_sweep<T, V, NT, TSTR, RSTR, TG>(bcode_s, d.n_bwd, c_s, xt, spt, tpt, rc);
                const unsigned mk = sentinel_mask();
                CUSR_FOR_V lsum += r[j] * r[j];
                if (p.jac) {
                    T *jrow = p.jac + (int64_t)wi.x * p.jac_kmax * p.N;
                    for (int k = 0; k < K; ++k) {
                        const VecT<T, V> g = *rc.at(k, rtab[k]);
                        CUSR_FOR_V if (valid[j]) jrow[(int64_t)k * p.N + si + j] = g.v[j];
                    }
                }
                // residual row; gradients of samples past N (only the last round of a tree's
                // last chunk has any) and of sentinel samples are zeroed
                *rc.at(K, rtab[K]) = pack<T, V>(r);
                if (si + V > p.N || mk) {
                    for (int k = 0; k < K; ++k) {
                        VecT<T, V> *q = rc.at(k, rtab[k]);
                        VecT<T, V> g = *q;
                        CUSR_FOR_V if (!valid[j] || ((mk >> j) & 1u)) g.v[j] = T(0);
                        *q = g;
                    }
                }
                __syncwarp();
                // the warp accumulates the (K+1)^2 Gram matrix of its 32 V samples as 8x8
                // fp64 tiles, four samples per product
                const T *tw = row_base + warp * 32 * V + (lane & 3);
#pragma unroll 2
                for (int s4 = 0; s4 < 32 * V; s4 += 4) {
                    double a[NTL];
#pragma unroll
                    for (int t = 0; t < NTL; ++t) a[t] = roff[t] >= 0 ? (double)tw[roff[t] + s4] : 0.0;
                    int c = 0;
#pragma unroll
                    for (int ti = 0; ti < NTL; ++ti) {
#pragma unroll
                        for (int tl = 0; tl <= ti; ++tl) dmma_884(cm[c++], a[ti], a[tl]);
                    }
                }
                // the next round's forward sweep overwrites these slots
                __syncwarp();
            }
        }

        // ---- block reduction of the item's sums (fixed order) -> partial slot ----
        const int P = GRAD ? nblock_size(K) : 1;
        T *dst = p.partials + d.p_off + (int64_t)wi.y * nblock_size(K);
        if (!grad) {
            lsum = warp_sum(lsum);
            if (lane == 0) red_s[warp] = lsum;
            __syncthreads();
            if (tid == 0) {
                T s = T(0);
#pragma unroll
                for (int w = 0; w < NW; ++w) s += red_s[w];
                dst[nblock_size(K) - 1] = s;
            }
        } else if constexpr (REV) {
            // packed (K+1)x(K+1) lower triangle == the partial layout (JtJ, Jtr, sum r^2)
            T *rw = red_s + warp * nblock_size(KC);
            const int grp = lane >> 2, q2 = 2 * (lane & 3);
            int c = 0;
#pragma unroll
            for (int ti = 0; ti < NTL; ++ti) {
#pragma unroll
                for (int tl = 0; tl <= ti; ++tl, ++c) {
                    const int i = 8 * ti + grp;
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq) {
                        const int l = 8 * tl + q2 + qq;
                        if (l <= i && i <= K) rw[i * (i + 1) / 2 + l] = (T)cm[c][qq];
                    }
                }
            }
            __syncthreads();
            for (int e = tid; e < P; e += NT) {
                T s = T(0);
#pragma unroll
                for (int w = 0; w < NW; ++w) s += red_s[w * nblock_size(KC) + e];
                dst[e] = s;
            }
        } else {
            T *rw = red_s + warp * nblock_size(KC);
#pragma unroll
            for (int i = 0; i < KC; ++i) {
                if (i < K) {
#pragma unroll
                    for (int l = 0; l <= i; ++l) {
                        const T v = warp_sum(acc[i * (i + 1) / 2 + l]);
                        if (lane == 0) rw[i * (i + 1) / 2 + l] = v;
                    }
                }
            }
            const int tri = K * (K + 1) / 2;
#pragma unroll
            for (int i = 0; i < KC; ++i) {
                if (i < K) {
                    const T v = warp_sum(jtr[i]);
                    if (lane == 0) rw[tri + i] = v;
                }
            }
            lsum = warp_sum(lsum);
            if (lane == 0) rw[tri + K] = lsum;
            __syncthreads();
            for (int e = tid; e < P; e += NT) {
                T s = T(0);
#pragma unroll
                for (int w = 0; w < NW; ++w) s += red_s[w * nblock_size(KC) + e];
                dst[e] = s;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------------
// Value-only pass: per-tree sum of squared residuals (and, optionally, per-sample values) at
// the given constants: the fp64 audit of fp32 fits and the value passes of the
// finite-difference Jacobian (K = 0 trees of a gradient launch take the fused kernel's
// value-and-loss path). Same items, shared-memory layout (the KC = 4
// class with a one-slot tape) and forward interpreter as the fused kernel, without tape,
// gradient or normal equations; writes the last entry of each item's partial slot.
// ---------------------------------------------------------------------------------------
template <typename T, int V, int NT, bool FAST>
__global__ void __launch_bounds__(NT) lm_value_kernel(const EvalParams<T> p) {
    typedef EvalSmem<T, V, NT, 4> L;
    constexpr int ROUND = NT * V;
    constexpr int NW = NT / 32;

    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_item;
    const L lay(p.code_cap, p.n_vars, p.spill_cap, 1, true);
    uint32_t *code_s = reinterpret_cast<uint32_t *>(smem + lay.code);
    T *c_s = reinterpret_cast<T *>(smem + lay.cval);
    VecF<V> *x_s = reinterpret_cast<VecF<V> *>(smem + lay.x);
    VecT<T, V> *spill_s = reinterpret_cast<VecT<T, V> *>(smem + lay.spill);
    T *red_s = reinterpret_cast<T *>(smem + lay.red);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_items = *p.n_items;
    VecF<V> *xt = x_s + tid;
    VecT<T, V> *spt = spill_s + tid;

    for (;;) {
        if (tid == 0) s_item = atomicAdd(p.counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= n_items) break;
        const int2 wi = p.items[it];
        const TreeDesc d = p.desc[wi.x];
        for (int i = tid; i < d.n_instr; i += NT) code_s[i] = p.code[d.code_off + i];
        if (tid == 0) code_s[d.n_instr] = 0u;   // prefetch pad
        for (int i = tid; i < d.K; i += NT) c_s[i] = p.c[d.c_off + i];
        __syncthreads();

        T lsum = T(0);
        const int64_t s0 = (int64_t)wi.y * p.chunk;
        const int64_t s_end = (int64_t)p.N < s0 + p.chunk ? (int64_t)p.N : s0 + p.chunk;
        const float *yrow = p.ym + d.y_off;
        for (int64_t base = s0; base < s_end; base += ROUND) {
            const int64_t si = base + (int64_t)tid * V;
            for (int v = 0; v < p.n_vars; ++v)
                xt[v * NT] = *reinterpret_cast<const VecF<V> *>(p.xs + (int64_t)v * p.ldx + si);
            const VecF<V> yv = *reinterpret_cast<const VecF<V> *>(yrow + si);
            T f[V];
            forward_sweep<T, V, NT, NT, false>(code_s, d.n_instr, c_s, xt, spt, nullptr, f);
            CUSR_FOR_V {
                const bool valid = si + j < p.N;
                const T r = valid ? f[j] - (T)yv.v[j] : T(0);
                lsum += r * r;
            }
            if (p.vals) {
                CUSR_FOR_V if (si + j < p.N) p.vals[(int64_t)wi.x * p.N + si + j] = f[j];
            }
        }
        lsum = warp_sum(lsum);
        if (lane == 0) red_s[warp] = lsum;
        __syncthreads();
        if (tid == 0) {
            T s = T(0);
#pragma unroll
            for (int w = 0; w < NW; ++w) s += red_s[w];
            p.partials[d.p_off + (int64_t)wi.y * nblock_size(d.K) + nblock_size(d.K) - 1] = s;
        }
        __syncthreads();
    }
}

}  // namespace cusr
