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
//   * persistent blocks of 128 threads pull work items from an atomic counter; items of a
//     bin are ordered most-expensive-tree first (LPT);
//   * every thread evaluates V consecutive samples at once (instruction decode is amortised
//     over V samples and the V chains give independent instructions);
//   * the tree program (warp-uniform) and the constants sit in shared memory; each thread's
//     spill stack, reverse tape, gradient rows and input row are private shared-memory
//     columns laid out [slot][thread] (conflict-free, no block barriers inside an item);
//   * the normal-equation sums for K <= 16 live in registers (KC = constant-count class,
//     rows >= K are skipped with warp-uniform branches); for K in 17..32 each warp builds the
//     (K+1)x(K+1) Gram matrix of [g; r] from a padded shared-memory tile, lanes owning
//     entries.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/cusr_co.h"
#include "program.h"
#include "ops.h"

namespace cusr {

constexpr int EVAL_THREADS = 128;
constexpr int EVAL_WARPS = EVAL_THREADS / 32;

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
    int chunk;               // samples per item (multiple of EVAL_THREADS * V)
    int n_vars;
    int code_cap;            // shared-memory words reserved for a program
    int spill_cap;           // spill slots reserved per thread
    int tape_cap;            // tape slots reserved per thread
    void *tape_g;            // global tape (TG instantiations): [block][tape_cap][thread]
    T *vals;                 // optional: per-sample values, [tree][N]
    T *jac;                  // optional: per-sample gradients, [tree][jac_kmax][N]
    int jac_kmax;
};

__host__ __device__ constexpr inline size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

// Shared-memory layout of one block; the host sizes the launch with the same function.
template <typename T, int V, int KC>
struct EvalSmem {
    static constexpr bool kBig = KC > 16;
    static constexpr int kGStride = EVAL_THREADS * V + (kBig ? 1 : 0);  // gradient row stride (T)
    static constexpr int kGRows = kBig ? KC + 1 : KC;                   // + residual row
    size_t code, cval, x, spill, tape, grad, red, total;
    __host__ __device__ EvalSmem(int code_cap, int n_vars, int spill_cap, int tape_cap,
                                 bool tape_in_smem = true) {
        size_t o = 0;
        code = o;  o += align16((size_t)code_cap * 4);
        cval = o;  o += align16((size_t)CO_MAX_K * sizeof(T));
        x = o;     o += align16((size_t)n_vars * EVAL_THREADS * V * 4);
        spill = o; o += align16((size_t)spill_cap * EVAL_THREADS * V * sizeof(T));
        tape = o;  o += tape_in_smem ? align16((size_t)tape_cap * EVAL_THREADS * V * sizeof(T)) : 0;
        grad = o;  o += align16((size_t)kGRows * kGStride * sizeof(T));
        red = o;   o += align16((size_t)EVAL_WARPS * nblock_size(KC) * sizeof(T));
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

// ---------------------------------------------------------------------------------------
// Forward sweep: value of the program at V samples; records the reverse tape when GRAD.
// ---------------------------------------------------------------------------------------
template <typename T, int V, bool GRAD>
__device__ __forceinline__ void forward_sweep(const uint32_t *__restrict__ code_s, int n_instr,
                                              const T *__restrict__ c_s,
                                              const VecF<V> *__restrict__ x_s,
                                              VecT<T, V> *__restrict__ spill_s,
                                              VecT<T, V> *__restrict__ tape_s, int tid,
                                              T (&tos)[V]) {
    typedef VecT<T, V> VT;
    for (int pc = 0; pc < n_instr; ++pc) {
        const uint32_t w = code_s[pc];
        const uint32_t op = w_op(w), mode = w_mode(w);
        if (op == OP_LOAD) {
            if (w_push(w)) {
                VT t; CUSR_FOR_V t.v[j] = tos[j];
                spill_s[w_sd(w) * EVAL_THREADS + tid] = t;
            }
            if (mode == M_VAR) {
                const VecF<V> xv = x_s[w_idx(w) * EVAL_THREADS + tid];
                CUSR_FOR_V tos[j] = (T)xv.v[j];
            } else {
                const T cv = c_s[w_idx(w)];
                CUSR_FOR_V tos[j] = cv;
            }
            continue;
        }
        if (op < OP_ADD) {
            T r[V], d[V];
            switch (op) {
#define CUSR_UN(OPC) case OPC: CUSR_FOR_V unary_op<T>(OPC, tos[j], r[j], d[j]); break;
                CUSR_UN(OP_SIN) CUSR_UN(OP_COS) CUSR_UN(OP_TAN) CUSR_UN(OP_SINH)
                CUSR_UN(OP_COSH) CUSR_UN(OP_TANH) CUSR_UN(OP_LOG) CUSR_UN(OP_LOGABS)
                CUSR_UN(OP_EXP) CUSR_UN(OP_INV) CUSR_UN(OP_NEG) CUSR_UN(OP_ABS)
                CUSR_UN(OP_SQRT) CUSR_UN(OP_SQRTABS)
#undef CUSR_UN
                default: CUSR_FOR_V { r[j] = T(0); d[j] = T(0); } break;
            }
            if (GRAD && op != OP_NEG && op != OP_UZERO) {
                VT t; CUSR_FOR_V t.v[j] = d[j];
                tape_s[w_ts(w) * EVAL_THREADS + tid] = t;
            }
            CUSR_FOR_V tos[j] = r[j];
            continue;
        }
        // binary: fetch the source operand
        T s[V];
        if (mode == M_VAR) {
            const VecF<V> xv = x_s[w_idx(w) * EVAL_THREADS + tid];
            CUSR_FOR_V s[j] = (T)xv.v[j];
        } else if (mode == M_CONST) {
            const T cv = c_s[w_idx(w)];
            CUSR_FOR_V s[j] = cv;
        } else {
            const VT t = spill_s[w_sd(w) * EVAL_THREADS + tid];
            CUSR_FOR_V s[j] = t.v[j];
        }
        const bool sw = w_swap(w);
        T o[V], dt[V], ds[V];
        switch (op) {
#define CUSR_BIN(OPC)                                                                    \
    case OPC:                                                                            \
        CUSR_FOR_V {                                                                     \
            T da, db;                                                                    \
            binary_op<T>(OPC, sw ? s[j] : tos[j], sw ? tos[j] : s[j], o[j], da, db);     \
            dt[j] = sw ? db : da; ds[j] = sw ? da : db;                                  \
        }                                                                                \
        break;
            CUSR_BIN(OP_ADD) CUSR_BIN(OP_SUB) CUSR_BIN(OP_MUL) CUSR_BIN(OP_DIV)
            CUSR_BIN(OP_POW) CUSR_BIN(OP_POWABS) CUSR_BIN(OP_MAX) CUSR_BIN(OP_MIN)
            CUSR_BIN(OP_LT) CUSR_BIN(OP_GT) CUSR_BIN(OP_LE) CUSR_BIN(OP_GE)
#undef CUSR_BIN
            default: CUSR_FOR_V { o[j] = T(0); dt[j] = T(0); ds[j] = T(0); } break;
        }
        if (GRAD) {
            const int ts = (int)w_ts(w);
            VT a, b;
            CUSR_FOR_V { a.v[j] = dt[j]; b.v[j] = ds[j]; }
            switch (op) {
                case OP_MUL:
                    if (mode == M_CONST) tape_s[ts * EVAL_THREADS + tid] = b;
                    else if (mode == M_POP) {
                        tape_s[ts * EVAL_THREADS + tid] = a;
                        tape_s[(ts + 1) * EVAL_THREADS + tid] = b;
                    }
                    break;
                case OP_DIV: case OP_POW: case OP_POWABS:
                    tape_s[ts * EVAL_THREADS + tid] = a;
                    if (mode != M_VAR) tape_s[(ts + 1) * EVAL_THREADS + tid] = b;
                    break;
                case OP_MAX: case OP_MIN:
                    tape_s[ts * EVAL_THREADS + tid] = a;
                    break;
                default: break;
            }
        }
        CUSR_FOR_V tos[j] = o[j];
    }
}

// gradient row access: [k][thread*V + j], rows padded in the cooperative (big-K) layout
template <typename T, int V, int GSTRIDE>
__device__ __forceinline__ void grad_put(T *__restrict__ g_s, int k, int tid, const T (&a)[V],
                                         bool unique) {
    T *row = g_s + k * GSTRIDE + tid * V;
    if (unique) {
        CUSR_FOR_V row[j] = a[j];
    } else {
        CUSR_FOR_V row[j] += a[j];
    }
}

// ---------------------------------------------------------------------------------------
// Reverse sweep: adjoints from the root to the leaves; grad row k receives df/dc_k.
// ---------------------------------------------------------------------------------------
template <typename T, int V, int GSTRIDE>
__device__ __forceinline__ void reverse_sweep(const uint32_t *__restrict__ code_s, int n_instr,
                                              const T *__restrict__ c_s,
                                              const VecF<V> *__restrict__ x_s,
                                              VecT<T, V> *__restrict__ spill_s,
                                              const VecT<T, V> *__restrict__ tape_s,
                                              T *__restrict__ g_s, int tid, bool unique) {
    typedef VecT<T, V> VT;
    T adj[V];
    CUSR_FOR_V adj[j] = T(1);
    for (int pc = n_instr - 1; pc >= 0; --pc) {
        const uint32_t w = code_s[pc];
        const uint32_t op = w_op(w), mode = w_mode(w);
        if (op == OP_LOAD) {
            if (mode == M_CONST) grad_put<T, V, GSTRIDE>(g_s, (int)w_idx(w), tid, adj, unique);
            if (w_push(w)) {
                const VT t = spill_s[w_sd(w) * EVAL_THREADS + tid];
                CUSR_FOR_V adj[j] = t.v[j];
            }
            continue;
        }
        if (op < OP_ADD) {
            if (op == OP_NEG) {
                CUSR_FOR_V adj[j] = -adj[j];
            } else if (op == OP_UZERO) {
                CUSR_FOR_V adj[j] = T(0);
            } else {
                const VT d = tape_s[w_ts(w) * EVAL_THREADS + tid];
                CUSR_FOR_V adj[j] = safe_mul(adj[j], d.v[j]);
            }
            continue;
        }
        const bool sw = w_swap(w);
        const int ts = (int)w_ts(w);
        T dt[V], ds[V];
        switch (op) {
            case OP_ADD: CUSR_FOR_V { dt[j] = T(1); ds[j] = T(1); } break;
            case OP_SUB: CUSR_FOR_V { dt[j] = sw ? T(-1) : T(1); ds[j] = -dt[j]; } break;
            case OP_MUL:
                if (mode == M_VAR) {
                    const VecF<V> xv = x_s[w_idx(w) * EVAL_THREADS + tid];
                    CUSR_FOR_V { dt[j] = (T)xv.v[j]; ds[j] = T(0); }
                } else if (mode == M_CONST) {
                    const T cv = c_s[w_idx(w)];
                    const VT b = tape_s[ts * EVAL_THREADS + tid];
                    CUSR_FOR_V { dt[j] = cv; ds[j] = b.v[j]; }
                } else {
                    const VT a = tape_s[ts * EVAL_THREADS + tid];
                    const VT b = tape_s[(ts + 1) * EVAL_THREADS + tid];
                    CUSR_FOR_V { dt[j] = a.v[j]; ds[j] = b.v[j]; }
                }
                break;
            case OP_DIV: case OP_POW: case OP_POWABS: {
                const VT a = tape_s[ts * EVAL_THREADS + tid];
                CUSR_FOR_V { dt[j] = a.v[j]; ds[j] = T(0); }
                if (mode != M_VAR) {
                    const VT b = tape_s[(ts + 1) * EVAL_THREADS + tid];
                    CUSR_FOR_V ds[j] = b.v[j];
                }
                break;
            }
            case OP_MAX: case OP_MIN: {
                const VT a = tape_s[ts * EVAL_THREADS + tid];
                CUSR_FOR_V { dt[j] = a.v[j]; ds[j] = T(1) - a.v[j]; }
                break;
            }
            default: CUSR_FOR_V { dt[j] = T(0); ds[j] = T(0); } break;
        }
        if (mode != M_VAR) {
            T as[V];
            CUSR_FOR_V as[j] = safe_mul(adj[j], ds[j]);
            if (mode == M_POP) {
                VT t; CUSR_FOR_V t.v[j] = as[j];
                spill_s[w_sd(w) * EVAL_THREADS + tid] = t;
            } else {
                grad_put<T, V, GSTRIDE>(g_s, (int)w_idx(w), tid, as, unique);
            }
        }
        CUSR_FOR_V adj[j] = safe_mul(adj[j], dt[j]);
    }
}

// ---------------------------------------------------------------------------------------
// The fused evaluation kernel.
//   T     arithmetic type (float / double)
//   V     samples per thread
//   TG    reverse tape in global scratch instead of shared memory
//   KC    constant-count class of the bin (trees with K <= KC)
//   GRAD  false: value and sum r^2 only (K = 0 trees never need more; the fp64 audit)
// ---------------------------------------------------------------------------------------
template <typename T, int V, int KC, bool GRAD, bool TG>
__global__ void __launch_bounds__(EVAL_THREADS)
lm_eval_kernel(const EvalParams<T> p) {
    typedef EvalSmem<T, V, KC> L;
    constexpr bool kBig = L::kBig;
    constexpr int GS = L::kGStride;
    constexpr int ROUND = EVAL_THREADS * V;
    constexpr int NTRI = KC * (KC + 1) / 2;
    constexpr int NACC = kBig ? (nblock_size(32) + 31) / 32 : 1;  // entries per lane (big-K)

    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_item;
    const L lay(p.code_cap, p.n_vars, p.spill_cap, p.tape_cap, !TG);
    uint32_t *code_s = reinterpret_cast<uint32_t *>(smem + lay.code);
    T *c_s = reinterpret_cast<T *>(smem + lay.cval);
    VecF<V> *x_s = reinterpret_cast<VecF<V> *>(smem + lay.x);
    VecT<T, V> *spill_s = reinterpret_cast<VecT<T, V> *>(smem + lay.spill);
    // reverse tape: private shared-memory columns, or (TG, trees whose tape would not fit
    // beside a second resident block) this block's slab of a global scratch buffer, read
    // back by the same thread and served from L1/L2
    VecT<T, V> *tape_s =
        TG ? reinterpret_cast<VecT<T, V> *>(p.tape_g) + (int64_t)blockIdx.x * p.tape_cap * EVAL_THREADS
           : reinterpret_cast<VecT<T, V> *>(smem + lay.tape);
    T *g_s = reinterpret_cast<T *>(smem + lay.grad);
    T *red_s = reinterpret_cast<T *>(smem + lay.red);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_items = *p.n_items;

    for (;;) {
        if (tid == 0) s_item = atomicAdd(p.counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= n_items) break;
        const int2 wi = p.items[it];
        const TreeDesc d = p.desc[wi.x];
        const int K = d.K;
        const bool unique = (d.flags & TD_UNIQUE_CONST) != 0;
        const bool grad = GRAD && K > 0;
        for (int i = tid; i < d.n_instr; i += EVAL_THREADS) code_s[i] = p.code[d.code_off + i];
        for (int i = tid; i < K; i += EVAL_THREADS) c_s[i] = p.c[d.c_off + i];
        __syncthreads();

        // accumulators (register path) / lane-owned Gram entries (big-K path)
        T acc[kBig ? 1 : (NTRI > 0 ? NTRI : 1)];
        T jtr[kBig ? 1 : KC];
        T lsum = T(0);
        T bacc[NACC];
        int boff_i[NACC], boff_l[NACC];
        if constexpr (!kBig) {
#pragma unroll
            for (int e = 0; e < NTRI; ++e) acc[e] = T(0);
#pragma unroll
            for (int e = 0; e < KC; ++e) jtr[e] = T(0);
        } else {
            // lane owns entries e = lane + 32u of the packed (K+1)x(K+1) lower triangle
            const int E = nblock_size(K);
#pragma unroll
            for (int u = 0; u < NACC; ++u) {
                bacc[u] = T(0);
                int e = lane + 32 * u, i = 0;
                if (e >= E) e = -1;
                if (e >= 0) { while ((i + 1) * (i + 2) / 2 <= e) ++i; }
                const int l = (e >= 0) ? e - i * (i + 1) / 2 : 0;
                boff_i[u] = (e >= 0) ? i * GS : -1;
                boff_l[u] = l * GS;
            }
        }

        const int64_t s0 = (int64_t)wi.y * p.chunk;
        const int64_t s_end = (int64_t)p.N < s0 + p.chunk ? (int64_t)p.N : s0 + p.chunk;
        const float *yrow = p.ym + d.y_off;
        for (int64_t base = s0; base < s_end; base += ROUND) {
            const int64_t si = base + (int64_t)tid * V;
            for (int v = 0; v < p.n_vars; ++v)
                x_s[v * EVAL_THREADS + tid] =
                    *reinterpret_cast<const VecF<V> *>(p.xs + (int64_t)v * p.ldx + si);
            const VecF<V> yv = *reinterpret_cast<const VecF<V> *>(yrow + si);

            T f[V];
            forward_sweep<T, V, GRAD>(code_s, d.n_instr, c_s, x_s, spill_s, tape_s, tid, f);
            T r[V];
            bool valid[V];
            CUSR_FOR_V {
                valid[j] = si + j < p.N;
                r[j] = valid[j] ? f[j] - (T)yv.v[j] : T(0);
                lsum += r[j] * r[j];
            }
            if (p.vals) {
                CUSR_FOR_V if (valid[j]) p.vals[(int64_t)wi.x * p.N + si + j] = f[j];
            }
            if (grad) {
                if (!unique) {
                    for (int k = 0; k < K; ++k) {
                        CUSR_FOR_V g_s[k * GS + tid * V + j] = T(0);
                    }
                }
                reverse_sweep<T, V, GS>(code_s, d.n_instr, c_s, x_s, spill_s, tape_s, g_s, tid,
                                        unique);
                if (p.jac) {
                    T *jrow = p.jac + (int64_t)wi.x * p.jac_kmax * p.N;
                    for (int k = 0; k < K; ++k) {
                        CUSR_FOR_V if (valid[j]) jrow[(int64_t)k * p.N + si + j] =
                            g_s[k * GS + tid * V + j];
                    }
                }
                if constexpr (!kBig) {
                    CUSR_FOR_V {
                        T g[KC];
#pragma unroll
                        for (int k = 0; k < KC; ++k)
                            if (k < K) g[k] = valid[j] ? g_s[k * GS + tid * V + j] : T(0);
#pragma unroll
                        for (int i = 0; i < KC; ++i) {
                            if (i < K) {
                                jtr[i] += g[i] * r[j];
#pragma unroll
                                for (int l = 0; l <= i; ++l) acc[i * (i + 1) / 2 + l] += g[i] * g[l];
                            }
                        }
                    }
                } else {
                    // stage the residual as row K, zero invalid samples' gradients
                    CUSR_FOR_V {
                        g_s[K * GS + tid * V + j] = r[j];
                        if (!valid[j])
                            for (int k = 0; k < K; ++k) g_s[k * GS + tid * V + j] = T(0);
                    }
                    __syncwarp();
                    const int sbase = warp * 32 * V;
                    for (int s = 0; s < 32 * V; ++s) {
#pragma unroll
                        for (int u = 0; u < NACC; ++u) {
                            if (boff_i[u] >= 0)
                                bacc[u] += g_s[boff_i[u] + sbase + s] * g_s[boff_l[u] + sbase + s];
                        }
                    }
                    __syncwarp();
                }
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
                for (int w = 0; w < EVAL_WARPS; ++w) s += red_s[w];
                dst[nblock_size(K) - 1] = s;
            }
        } else if constexpr (!kBig) {
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
            for (int e = tid; e < P; e += EVAL_THREADS) {
                T s = T(0);
#pragma unroll
                for (int w = 0; w < EVAL_WARPS; ++w) s += red_s[w * nblock_size(KC) + e];
                dst[e] = s;
            }
        } else {
            T *rw = red_s + warp * nblock_size(KC);
#pragma unroll
            for (int u = 0; u < NACC; ++u)
                if (boff_i[u] >= 0) rw[lane + 32 * u] = bacc[u];
            __syncthreads();
            for (int e = tid; e < P; e += EVAL_THREADS) {
                T s = T(0);
#pragma unroll
                for (int w = 0; w < EVAL_WARPS; ++w) s += red_s[w * nblock_size(KC) + e];
                dst[e] = s;
            }
        }
        __syncthreads();
    }
}

}  // namespace cusr
