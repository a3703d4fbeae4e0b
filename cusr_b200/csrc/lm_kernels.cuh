// lm_kernels.cuh — per-tree LM bookkeeping on the device: accept / reject / lambda /
// convergence of the evaluated trial, the damped Cholesky solve of the next step, the work
// list of the next evaluation, and the fp64 audit.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "program.h"
#include "eval_kernel.cuh"
#include "warp_linalg.cuh"

namespace cusr {

// internal per-tree status: RUNNING while iterating, else the final STATUS_* code
constexpr int32_t ST_RUNNING = -1;

template <typename T>
struct StepParams {
    const TreeDesc *desc;
    int M;
    const T *partials;       // per-item sums of the last evaluation
    T *blk;                  // normal-equation block at the accepted point, q_off
    T *c;                    // accepted constants
    T *ctry;                 // trial constants (evaluated point)
    T *delta;                // last solved step
    T *lam;                  // Marquardt damping
    T *loss;                 // accepted 0.5*sum r^2
    T *loss_init;
    int32_t *status;
    int32_t *iters;
    int32_t *pending;        // 1: the tree's trial was evaluated by the last pass
    int32_t *n_eval;         // evaluations consumed per tree (initial pass + trials)
    const T *reduced;        // sample-sharded mode: per-tree sums all-reduced over ranks
                             // (q_off layout, replaces the chunk partials), else null
    double damping_floor;    // 0: reference damping diag * (1 + lam)
    int damping_always;      // with a floor: floored damping on every solve (else fallback)
    const uint8_t *imode;    // per fit (start axis, IM_* below), or null: every fit uses the
                             // reference schedule with the call's damping settings
    int *n_running;          // trees still running after this step (early exit)
    int max_iter;            // LM iterations per fit
    int fd_order;            // the FD variant's acceptance order (co_lib.cu:456-471)
    T xtol;
};

// per-fit mode bits (the start axis): the trust-region algorithm (run by lm_tr_step_kernel,
// skipped here), and the floored damping on every solve for a reference-schedule fit
constexpr uint8_t IM_TR = 1;
constexpr uint8_t IM_DAMP_ALWAYS = 2;
// a trust-region fit whose normal equations are formed and factored in double-double
// (dd_gram_kernel, lm_tr_step_kernel_dd): fp64 fits with CoOptions.tr_dd
constexpr uint8_t IM_TR_DD = 8;

constexpr int STEP_THREADS = 256;
constexpr int STEP_WARPS = STEP_THREADS / 32;
// per-warp shared memory (doubles): sums [561 T] + the damped system (K rows of WL_LD)
constexpr int STEP_SUMS_D = 576;
constexpr int STEP_WARP_D = STEP_SUMS_D + CO_MAX_K * WL_LD;

// Lane i < K of a warp writes row i of the damped system's lower triangle (packed block b):
// a_il = JtJ_il, the diagonal damped by diag * (1 + lam) (batch_lm_ad.cu:152-159) or, with
// `floored`, by diag + lam * max(diag, fl) (fl = damping floor * the largest diagonal).
template <typename T>
__device__ __forceinline__ void step_build_rows(double *W, const T *b, int K, int lane,
                                                double lam, double fac, bool floored,
                                                double floor_frac) {
    double dg = 0.0;
    if (lane < K) {
        const T *row = b + lane * (lane + 1) / 2;
        for (int l = 0; l <= lane; ++l) W[lane * WL_LD + l] = (double)row[l];
        dg = W[lane * WL_LD + lane];
    }
    if (floored) {
        const double fl = wl_max(dg) * floor_frac;
        if (lane < K) W[lane * WL_LD + lane] = dg + lam * (dg > fl ? dg : fl);
    } else if (lane < K) {
        W[lane * WL_LD + lane] = dg * fac;
    }
    __syncwarp();
}

// One warp per tree. Mirrors the reference LM iteration (co_lib.cu:343-483 with the AD
// ordering of :438-455, batch_lm_revad.cu:396-500):
//   finalize the evaluated trial: non-finite loss -> FAIL_NAN; loss_try <= loss -> accept
//   (c, loss, JtJ, Jtr move to the trial), then |delta| < xtol(|c_try| + xtol) -> CONVERGED,
//   else lambda = max(0.1 lambda, 1e-12); otherwise reject, lambda *= 10, > 1e12 -> FAIL_NAN;
//   solve: A = JtJ with diag *= (1 + lambda) (batch_lm_ad.cu:152-159), Cholesky in fp64
//   (the reference's SOLVE_FP64 form), s <= 0 -> this iteration is a rejected step,
//   lambda *= 10, > 1e12 -> FAIL_CHOLESKY; else c_try = c + delta is queued for evaluation.
// The J/JtJ/Jtr of an accepted trial were built by the same pass that computed its loss, so
// an accept needs no re-evaluation and a reject re-solves from the stored block.
// Lane 0 keeps the per-tree bookkeeping; the K-vectors and the factorisation are spread over
// the lanes (lane i: constant i, row i of the system), so a K = 32 solve takes O(K^2) warp
// steps (wl_chol_left: the reference's serial operation order per element).
template <typename T>
__global__ void __launch_bounds__(STEP_THREADS) lm_step_kernel(const StepParams<T> p) {
    extern __shared__ double step_sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    T *sums = reinterpret_cast<T *>(step_sm + warp * STEP_WARP_D);
    double *W = step_sm + warp * STEP_WARP_D + STEP_SUMS_D;
    for (int m = blockIdx.x * STEP_WARPS + warp; m < p.M; m += gridDim.x * STEP_WARPS) {
        int st = p.status[m];
        if (st != ST_RUNNING) continue;
        const uint8_t mode = p.imode ? p.imode[m] : 0;
        if (mode & IM_TR) continue;
        const TreeDesc d = p.desc[m];
        const int K = d.K, P = nblock_size(K);
        const int pend = p.pending[m];
        // the first evaluation of a fit is at its start point (c_init for start 0)
        const bool initial = p.n_eval[m] == 0;
        __syncwarp();
        if (pend) {
            if (p.reduced) {
                for (int e = lane; e < P; e += 32) sums[e] = p.reduced[d.q_off + e];
            } else {
                for (int e = lane; e < P; e += 32) {
                    const T *src = p.partials + d.p_off + e;
                    T s = T(0);
                    for (int ch = 0; ch < d.n_chunks; ++ch) s += src[(int64_t)ch * P];
                    sums[e] = s;
                }
            }
        }
        // |delta|^2 and |c_try|^2 of the evaluated trial, lane k holding constant k
        const bool trial = pend && !initial;
        T ck = T(0), dn2 = T(0), cn2 = T(0);
        if (trial) {
            T dk = T(0);
            if (lane < K) {
                dk = p.delta[d.c_off + lane];
                ck = p.ctry[d.c_off + lane];
            }
            dn2 = wl_sum_t(dk * dk);
            cn2 = wl_sum_t(ck * ck);
        }
        __syncwarp();
        int accept = 0;
        T lam = T(0);
        if (lane == 0) {
            lam = p.lam[m];
            if (pend) {
                p.pending[m] = 0;
                p.n_eval[m] += 1;
                const T ltry = T(0.5) * sums[P - 1];
                if (initial) {
                    p.loss_init[m] = ltry;
                    p.loss[m] = ltry;
                    accept = 1;
                    if (K == 0) st = STATUS_K0_SKIP;
                    else if (!Mth<T>::finite(ltry)) st = STATUS_FAIL_NAN;
                } else {
                    p.iters[m] += 1;
                    if (!Mth<T>::finite(ltry)) {
                        st = STATUS_FAIL_NAN;
                    } else {
                        const T dn = Mth<T>::sqrt(dn2), cn = Mth<T>::sqrt(cn2);
                        const bool small = dn < p.xtol * (cn + p.xtol);
                        // FD variant: a small step converges (and is kept) first, then a
                        // strict improvement is accepted; AD: improvement first
                        const bool better = p.fd_order ? (small || ltry < p.loss[m])
                                                       : ltry <= p.loss[m];
                        if (better) {
                            accept = 1;
                            p.loss[m] = ltry;
                            if (small) {
                                st = STATUS_CONVERGED;
                            } else {
                                lam *= T(0.1);
                                if (lam < T(1e-12)) lam = T(1e-12);
                            }
                        } else {
                            lam *= T(10);
                            if (lam > T(1e12)) st = STATUS_FAIL_NAN;
                        }
                    }
                }
            }
            // every running fit takes one LM iteration per pass (an evaluated trial or a
            // factorisation failure); after max_iter of them it stops
            if (st == ST_RUNNING && p.iters[m] >= p.max_iter) st = STATUS_MAXITER;
        }
        accept = __shfl_sync(0xffffffffu, accept, 0);
        st = __shfl_sync(0xffffffffu, st, 0);
        lam = __shfl_sync(0xffffffffu, lam, 0);
        if (accept) {
            for (int e = lane; e < P; e += 32) p.blk[d.q_off + e] = sums[e];
            if (trial && lane < K) p.c[d.c_off + lane] = ck;
        }
        if (st == ST_RUNNING) {
            // the accepted point's block: this pass's sums after an accept, else the stored one
            const T *b = accept ? sums : p.blk + d.q_off;
            const int tri = K * (K + 1) / 2;
            const double fac = (double)(T(1) + lam);
            const bool always = p.damping_floor > 0.0 &&
                                (p.damping_always || (mode & IM_DAMP_ALWAYS));
            step_build_rows(W, b, K, lane, (double)lam, fac, always, p.damping_floor);
            bool ok = wl_chol_left(W, K, lane);
            // robust mode: a system the reference damping cannot factor (a zero or
            // negligible Jacobian column) is retried with the damping floor
            if (!ok && p.damping_floor > 0.0 && !always) {
                step_build_rows(W, b, K, lane, (double)lam, fac, true, p.damping_floor);
                ok = wl_chol_left(W, K, lane);
            }
            if (!ok) {
                if (lane == 0) {
                    p.iters[m] += 1;
                    lam *= T(10);
                    if (lam > T(1e12)) st = STATUS_FAIL_CHOLESKY;
                }
            } else {
                const double y = wl_fsub(W, K, lane, lane < K ? -(double)b[tri + lane] : 0.0);
                const double x = wl_bsub(W, K, lane, y);
                if (lane < K) {
                    const T dk = (T)x;
                    p.delta[d.c_off + lane] = dk;
                    p.ctry[d.c_off + lane] = p.c[d.c_off + lane] + dk;
                }
                if (lane == 0) p.pending[m] = 1;
            }
        }
        if (lane == 0) {
            p.lam[m] = lam;
            p.status[m] = st;
            if (st == ST_RUNNING) atomicAdd(p.n_running, 1);
        }
        __syncwarp();
    }
}

// Work list of one bin: every chunk of every pending tree, bin order (most expensive
// first). One block per bin; also resets the bin's work counter.
struct ItemsParams {
    const TreeDesc *desc;
    const int32_t *bin_trees;      // concatenated per-bin tree lists
    const int64_t *bin_tree_off;   // [n_bins + 1]
    const int64_t *bin_item_off;   // [n_bins]
    const int32_t *pending;
    int2 *items;
    int *n_items;                  // [n_bins]
    int *counter;                  // [n_bins]
};

constexpr int ITEMS_THREADS = 1024;

__global__ void __launch_bounds__(ITEMS_THREADS) build_items_kernel(const ItemsParams p) {
    __shared__ int warp_tot[ITEMS_THREADS / 32];
    __shared__ int s_run;
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t t0 = p.bin_tree_off[b], t1 = p.bin_tree_off[b + 1];
    int2 *items = p.items + p.bin_item_off[b];
    if (tid == 0) s_run = 0;
    __syncthreads();
    for (int64_t base = t0; base < t1; base += ITEMS_THREADS) {
        const int64_t ti = base + tid;
        int tree = -1, cnt = 0;
        if (ti < t1) {
            tree = p.bin_trees[ti];
            cnt = p.pending[tree] ? p.desc[tree].n_chunks : 0;
        }
        // block exclusive scan of cnt
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int v = warp_tot[lane];
            int inc = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += u;
            }
            warp_tot[lane] = inc - v;   // exclusive warp offsets
        }
        __syncthreads();
        const int off = s_run + warp_tot[warp] + incl - cnt;
        for (int c = 0; c < cnt; ++c) items[off + c] = make_int2(tree, c);
        __syncthreads();
        if (tid == ITEMS_THREADS - 1) s_run = off + cnt;
        __syncthreads();
    }
    if (tid == 0) {
        p.n_items[b] = s_run;
        p.counter[b] = 0;
    }
}

// SoA transpose of the inputs: xs [N][n_vars] (pop.bin) -> [n_vars][ldx], zero padded.
__global__ void transpose_x_kernel(const float *__restrict__ xs, int64_t N, int n_vars,
                                   int64_t ldx, float *__restrict__ out) {
    const int64_t total = (int64_t)n_vars * ldx;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = e / ldx, i = e - v * ldx;
        out[e] = (i < N) ? xs[i * n_vars + v] : 0.0f;
    }
}

// Evaluation entry: constants of the evaluated point (fp64 from the caller), every tree pending.
template <typename T>
__global__ void load_point_kernel(const double *__restrict__ c64, int64_t total_c, T *c, int M,
                                  int32_t *pending) {
    const int64_t gs = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total_c; i += gs)
        c[i] = (T)c64[i];
    for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < M; m += gs)
        pending[m] = 1;
}

// Finite-difference Jacobian, column k (the reference FD variant, batch_lm_ad.cu:95-132):
// every tree with K > k gets c_k + h with h = eps * |c_k| (eps when c_k == 0), the step taken
// as the representable difference (c_k + h) - c_k (eps again if that is 0); the other
// constants stay. Trees with K <= k are not evaluated (pending = 0).
template <typename T>
__global__ void fd_perturb_kernel(const TreeDesc *desc, int M, const T *c, int k, T eps,
                                  T *c_out, T *h_out, int32_t *pending) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const TreeDesc d = desc[m];
        for (int t = 0; t < d.K; ++t) c_out[d.c_off + t] = c[d.c_off + t];
        T h = T(0);
        if (k < d.K) {
            const T saved = c[d.c_off + k];
            h = eps * (saved < T(0) ? -saved : saved);
            if (h == T(0)) h = eps;
            const T cp = saved + h;
            h = cp - saved;
            if (h == T(0)) h = eps;
            c_out[d.c_off + k] = cp;
        }
        h_out[m] = h;
        pending[m] = k < d.K ? 1 : 0;
    }
}

// J[m][k][i] = (f_k(x_i) - f(x_i)) / h_m for the trees with K > k (IEEE division).
template <typename T>
__global__ void fd_column_kernel(const TreeDesc *desc, int M, int N, int k, int kmax,
                                 const T *vals_k, const T *vals_0, const T *h, T *jac) {
    const int64_t total = (int64_t)M * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(e / N);
        if (k >= desc[m].K) continue;
        const int64_t i = e - (int64_t)m * N;
        jac[((int64_t)m * kmax + k) * N + i] = (vals_k[e] - vals_0[e]) / h[m];
    }
}

// Per-tree sums of the chunk partials for populations with many chunks per tree (the
// sample-sharded all-reduce input, and the step kernels' input when N spans hundreds of
// chunks): one block per tree (grid-stride over trees), its warps take interleaved chunk
// slices and its lanes 32 consecutive elements (coalesced reads of a chunk's partial row);
// the slice sums of an element are then added in slice order, a fixed order, so the sums are
// the same run to run. Raw sums (the step kernel halves the loss element itself).
constexpr int CSUM_THREADS = 256;
template <typename T>
__global__ void __launch_bounds__(CSUM_THREADS)
chunk_sum_kernel(const TreeDesc *desc, int M, const T *partials, T *out) {
    constexpr int NW = CSUM_THREADS / 32;
    __shared__ T part[NW][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = blockIdx.x; m < M; m += gridDim.x) {
        const TreeDesc d = desc[m];
        const int P = nblock_size(d.K);
        for (int e0 = 0; e0 < P; e0 += 32) {
            const int e = e0 + lane;
            T s = T(0);
            if (e < P)
                for (int ch = warp; ch < d.n_chunks; ch += NW)
                    s += partials[d.p_off + (int64_t)ch * P + e];
            part[warp][lane] = s;
            __syncthreads();
            if (warp == 0 && e < P) {
                T t = part[0][lane];
#pragma unroll
                for (int w = 1; w < NW; ++w) t += part[w][lane];
                out[d.q_off + e] = t;
            }
            __syncthreads();
        }
    }
}

// Per-tree normal-equation block = sum of its chunk partials in chunk order.
template <typename T>
__global__ void sum_blocks_kernel(const TreeDesc *desc, int M, const T *partials, T *blk) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const TreeDesc d = desc[m];
        const int P = nblock_size(d.K);
        for (int e = 0; e < P; ++e) {
            T s = T(0);
            for (int ch = 0; ch < d.n_chunks; ++ch) s += partials[d.p_off + (int64_t)ch * P + e];
            blk[d.q_off + e] = (e == P - 1) ? T(0.5) * s : s;
        }
    }
}

// Peak-throughput probes: independent FMA chains per thread (no memory traffic in the loop).
template <typename T>
__global__ void fma_probe_kernel(T *out, int iters, T b, T c) {
    T a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = (T)(threadIdx.x + i);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = a[i] * b + c;
    }
    T s = T(0);
#pragma unroll
    for (int i = 0; i < 16; ++i) s += a[i];
    if (s == T(-1.2345)) out[0] = s;   // keeps the chains alive
}

// ---- fp64 honesty audit (lm_core.cuh:299-351) -------------------------------------------
// Trees whose fp64 loss at the delivered constants is non-finite or worse than at c_init
// are reverted to c_init, a CONVERGED status becomes MAXITER, and the reported final loss
// becomes the fp64 loss at c_init.
// Fits that never ran (later-wave starts a tree retired) are not evaluated.
__global__ void audit_prepare_kernel(const TreeDesc *desc, int M, const float *c_now,
                                     int64_t total_c, double *c64, int32_t *pending,
                                     const int32_t *n_eval) {
    const int64_t gs = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total_c; i += gs)
        c64[i] = (double)c_now[i];
    for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < M; m += gs)
        pending[m] = (desc[m].K > 0 && n_eval[m] > 0) ? 1 : 0;
}

__global__ void audit_loss_kernel(const TreeDesc *desc, int M, const double *partials,
                                  double *loss64) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const TreeDesc d = desc[m];
        if (d.K == 0) { loss64[m] = 0.0; continue; }
        const int P = nblock_size(d.K);
        double s = 0.0;
        for (int ch = 0; ch < d.n_chunks; ++ch) s += partials[d.p_off + (int64_t)ch * P + P - 1];
        loss64[m] = 0.5 * s;
    }
}

template <typename T>
__global__ void audit_apply_kernel(const TreeDesc *desc, int M, const double *lfinal,
                                   const double *linit, const float *c_init, T *c, T *loss,
                                   int32_t *status, const int32_t *n_eval, int *n_reverted) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const TreeDesc d = desc[m];
        if (d.K == 0 || n_eval[m] == 0) continue;
        const double lf = lfinal[m], li = linit[m];
        if (!isfinite(lf) || (isfinite(li) && lf > li)) {
            for (int k = 0; k < d.K; ++k) c[d.c_off + k] = (T)c_init[d.c_off + k];
            if (status[m] == STATUS_CONVERGED) status[m] = ST_RUNNING;   // reported as MAXITER
            loss[m] = (T)li;
            atomicAdd(n_reverted, 1);
        }
    }
}

}  // namespace cusr
