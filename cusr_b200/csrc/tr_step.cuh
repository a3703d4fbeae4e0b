// tr_step.cuh — the trust-region Levenberg–Marquardt step (Moré 1977, "The Levenberg-
// Marquardt algorithm: implementation and theory"; the algorithm of MINPACK's lmder, which
// the reference's CPU backend runs through scipy.optimize.least_squares(method='lm'),
// cusr/benchmark/backends.py:97-120), one warp per fit, on the normal equations the fused
// evaluation pass already produces.
//
// Per fit the state is the scaling D (per constant), the trust radius Delta, the LM parameter
// par, |f| at the accepted point, |D x| and |D p| of the last step. After each evaluated trial:
//   actred = 1 - (|f_try| / |f|)^2 (-1 when |f_try| >= 10 |f|), prered = (|J p|^2 +
//   2 par |D p|^2) / |f|^2, ratio = actred / prered; ratio <= 1/4 shrinks Delta (by the
//   directional-derivative factor, within [1/10, 1/2]), ratio >= 3/4 (or par = 0) sets
//   Delta = 2 |D p|; ratio >= 1e-4 accepts the trial (its J, J^T f, |f|^2 become current,
//   since the pass evaluated them at the trial point); convergence: |actred| <= ftol and
//   prered <= ftol, or Delta <= xtol |D x|, or at the next accepted point
//   max_j |(J^T f)_j| / (|f| |J_j|) <= gtol; D_j = max(D_j, |J_j|).
// The step p solves (J^T J + par D^2) p = -J^T f with par chosen so that | |D p| - Delta | <=
// Delta / 10 (or par = 0 when the Gauss-Newton step is inside the region): Newton iteration on
// 1 / |D p| - 1 / Delta with the safeguards [parl, paru] and at most 10 factorisations.
// MINPACK works on the QR factors of J; here the same equations are solved through Cholesky
// factors of J^T J + par D^2 (the Gram matrix of the pass, accumulated in fp64): lanes own rows,
// right-looking updates, so a K <= 32 factorisation takes O(K^2) warp steps. The Gauss-Newton
// step uses symmetric (diagonal) pivoting, which orders the columns as QR column pivoting does,
// and stops at the first non-positive pivot: a rank-deficient J gives the basic solution on
// the independent columns (MINPACK's QR keeps rounding-size pivots there instead).
#pragma once
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>
#include "lm_kernels.cuh"
#include "warp_linalg.cuh"

namespace cusr {

// per-fit state of the trust-region algorithm (fp64), in TrParams::tr
enum TrField { TR_DELTA = 0, TR_PAR, TR_FNORM, TR_XNORM, TR_PNORM, TR_GNORM, TR_FIELDS };

template <typename T>
struct TrParams {
    const TreeDesc *desc;
    int M;
    const T *partials;
    T *blk, *c, *ctry, *delta, *loss, *loss_init;
    int32_t *status, *iters, *pending, *n_eval;
    const uint8_t *imode;
    double *tr;          // [M][TR_FIELDS]
    double *diag;        // per constant (TreeDesc::c_off)
    int32_t *outer;      // outer iterations (accepted points) per fit
    int *n_running;
    int max_nfev;        // evaluations per fit, the initial one included
    double ftol, xtol, gtol, factor;
    const double *ddg = nullptr;   // double-double sums of the pass (dd_gram_kernel), or null
    double *blk_dd = nullptr;      // double-double block at the accepted point (IM_TR_DD fits)
};

constexpr int TR_THREADS = 128;
constexpr int TR_WARPS = TR_THREADS / 32;
constexpr int TR_THREADS_DD = 64;     // the double-double variant: twice the shared memory
// per warp, in scalars S: the factorisation workspace W (K x K); the summed block of the pass
// (at most 561 values) shares its space: it is read (loss, finiteness, the accepted block)
// before the step's factorisations write W. J^T J itself is read from the accepted block in
// global memory (TrA).
constexpr int TR_WARP_D = CO_MAX_K * WL_LD;
static_assert(CO_MAX_K * WL_LD >= nblock_size(CO_MAX_K), "the block fits in W");
template <typename S> __host__ __device__ constexpr int tr_threads() {
    return sizeof(S) == 8 ? TR_THREADS : TR_THREADS_DD;
}

// Symmetrically pivoted Cholesky of W = A (full, lanes own rows): at step b the largest
// remaining diagonal is the pivot perm[b]; the column values l_i are kept in W[i][perm[b]].
// Returns the rank r (pivots taken before the first non-positive one).
template <typename S>
__device__ int tr_pchol(S *W, int K, int lane, int *perm) {
    bool done = lane >= K;
    int r = 0;
    for (int b = 0; b < K; ++b) {
        __syncwarp();
        S v = done ? S(-1.0) : W[lane * WL_LD + lane];
        int p = lane;
        // argmax with ties to the lower index: every lane ends with the same (v, p)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const S v2 = shfl_xor(v, o);
            const int p2 = __shfl_xor_sync(0xffffffffu, p, o);
            if (v2 > v || (v2 == v && p2 < p)) { v = v2; p = p2; }
        }
        if (!(v > S(0.0))) break;
        const S lpp = sqrt(v);
        S li = S(0.0);
        if (!done && lane != p) li = W[lane * WL_LD + p] / lpp;
        __syncwarp();
        if (!done && lane != p) W[lane * WL_LD + p] = li;
        if (lane == p) { W[p * WL_LD + p] = lpp; done = true; }
        if (lane == 0) perm[b] = p;
        // trailing update of the rows and columns still remaining
        const bool act = !done;
        for (int k = 0; k < K; ++k) {
            const S lk = shfl(li, k);
            const int dk = __shfl_sync(0xffffffffu, (int)done, k);
            if (act && !dk) W[lane * WL_LD + k] -= li * lk;
        }
        ++r;
    }
    __syncwarp();
    return r;
}

// Gauss-Newton step on the pivoted factor: x = -(A^+) g on the r independent columns,
// 0 on the others (lane i holds g_i, returns x_i). Lanes work in pivot order: lane a takes
// row perm[a]; L[a][k] = W[perm[a]][perm[k]].
template <typename S>
__device__ S tr_gn_step(const S *W, int r, int lane, const int *perm, S g) {
    const int pa = lane < r ? perm[lane] : 0;
    S b = shfl(-g, pa);
    if (lane >= r) b = S(0.0);
    S y = S(0.0);
    for (int k = 0; k < r; ++k) {          // forward: L y = b
        const int pk = perm[k];
        S yk = S(0.0);
        if (lane == k) yk = b / W[pk * WL_LD + pk];
        yk = shfl(yk, k);
        if (lane == k) y = yk;
        if (lane > k && lane < r) b -= W[pa * WL_LD + pk] * yk;
    }
    S z = S(0.0);
    for (int k = r - 1; k >= 0; --k) {     // back: L^T z = y
        const int pk = perm[k];
        S zk = S(0.0);
        if (lane == k) zk = y / W[pk * WL_LD + pk];
        zk = shfl(zk, k);
        if (lane == k) z = zk;
        if (lane < k) y -= W[pk * WL_LD + pa] * zk;
    }
    // back to the original order: lane i takes z of the pivot position holding i
    S x = S(0.0);
    for (int a = 0; a < r; ++a) {
        const S za = shfl(z, a);
        if (lane == perm[a]) x = za;
    }
    return x;
}

// forward solve with the full-rank pivoted factor (L w = v[perm]), returns |w|
template <typename S>
__device__ double tr_pfsub_norm(const S *W, int K, int lane, const int *perm, S v) {
    const int pa = lane < K ? perm[lane] : 0;
    S b = shfl(v, pa);
    if (lane >= K) b = S(0.0);
    S w = S(0.0);
    for (int k = 0; k < K; ++k) {
        const int pk = perm[k];
        S wk = S(0.0);
        if (lane == k) wk = b / W[pk * WL_LD + pk];
        wk = shfl(wk, k);
        if (lane == k) w = wk;
        if (lane > k && lane < K) b -= W[pa * WL_LD + pk] * wk;
    }
    return wl_norm(w);
}

// J^T J of the accepted point, read from its packed lower-triangle block in global memory
// (T values, or (hi, lo) pairs for double-double fits); the block is read where it is needed
// instead of being kept in shared memory, so more warps stay resident
template <typename T, typename S>
struct TrA {
    const T *blk;          // packed block of the fit (its q_off applied)
    const double *blk_dd;  // the same as (hi, lo) pairs, double-double fits
    __device__ __forceinline__ S operator()(int i, int l) const {
        const int hi = i > l ? i : l, lo = i > l ? l : i;
        const int e = hi * (hi + 1) / 2 + lo;
        if constexpr (sizeof(S) == 16) return S(blk_dd[2 * e], blk_dd[2 * e + 1]);
        else return S((double)blk[e]);
    }
};

// W = A + par diag(d^2), rows owned by lanes
template <typename S, typename AV>
__device__ __forceinline__ void tr_load(S *W, const AV A, int K, int lane, double par,
                                        double d) {
    if (lane < K) {
        for (int k = 0; k < K; ++k) W[lane * WL_LD + k] = A(lane, k);
        W[lane * WL_LD + lane] += S(par * d * d);
    }
    __syncwarp();
}

// The LM parameter and step for trust radius delta (MINPACK lmpar, on normal equations).
// Lane i holds g_i = (J^T f)_i and d_i; returns x_i (the step) and updates par.
template <typename S, typename AV>
__device__ __forceinline__ S tr_lmpar(const AV A, S *W, int *perm, int K, int lane, S g, double d,
                      double delta, double &par) {
    const double dwarf = DBL_MIN;
    // Gauss-Newton direction
    tr_load(W, A, K, lane, 0.0, d);
    const int r = tr_pchol(W, K, lane, perm);
    S x = r > 0 ? tr_gn_step(W, r, lane, perm, g) : S(0.0);
    if (lane >= K) x = S(0.0);
    double dxnorm = wl_norm(S(d) * x);
    double fp = dxnorm - delta;
    if (fp <= 0.1 * delta) {
        par = 0.0;
        return x;
    }
    // lower bound (J of full rank): the Newton step of 1/|Dx| - 1/delta at par = 0
    double parl = 0.0;
    if (r == K) {
        const S v = lane < K ? S(d) * (S(d) * x) / S(dxnorm) : S(0.0);
        const double t = tr_pfsub_norm(W, K, lane, perm, v);
        parl = ((fp / delta) / t) / t;
    }
    // upper bound
    const double gnorm = wl_norm(lane < K ? g / S(d) : S(0.0));
    double paru = gnorm / delta;
    if (paru == 0.0) paru = dwarf / fmin(delta, 0.1);
    par = fmax(par, parl);
    par = fmin(par, paru);
    if (par == 0.0) par = gnorm / dxnorm;
    for (int iter = 1;; ++iter) {
        if (par == 0.0) par = fmax(dwarf, 0.001 * paru);
        tr_load(W, A, K, lane, par, d);
        // a system that rounding left indefinite (dependent columns, par tiny against the
        // scale of J^T J) is factored with par raised until it is positive definite
        int guard = 0;
        while (!wl_chol(W, K, lane) && guard < 64) {
            const double amax = to_double(wl_max(lane < K ? fabs(A(lane, lane)) : S(0.0)));
            const double dmin = -wl_max(lane < K ? -(d * d) : -DBL_MAX);
            par = fmax(fmax(2.0 * par, 1e-15 * amax / dmin), dwarf);
            tr_load(W, A, K, lane, par, d);
            ++guard;
        }
        const S y = wl_fsub(W, K, lane, lane < K ? -g : S(0.0));
        x = wl_bsub(W, K, lane, y);
        if (lane >= K) x = S(0.0);
        dxnorm = wl_norm(S(d) * x);
        const double temp = fp;
        fp = dxnorm - delta;
        if (fabs(fp) <= 0.1 * delta || (parl == 0.0 && fp <= temp && temp < 0.0) || iter == 10)
            return x;
        const S v = lane < K ? S(d) * (S(d) * x) / S(dxnorm) : S(0.0);
        const double t = wl_norm(wl_fsub(W, K, lane, v));
        const double parc = ((fp / delta) / t) / t;
        if (fp > 0.0) parl = fmax(parl, par);
        if (fp < 0.0) paru = fmin(paru, par);
        par = fmax(parl, par + parc);
    }
}

// One trust-region step for every running fit of mode IM_TR whose trial was evaluated. S is
// the scalar of the normal equations: double (lm_tr_step_kernel), or double-double for the
// IM_TR_DD fits (lm_tr_step_kernel_dd: sums from dd_gram_kernel, accepted block in blk_dd).
template <typename T, typename S>
__global__ void __launch_bounds__(tr_threads<S>()) lm_tr_step_kernel_s(const TrParams<T> p) {
    constexpr bool DDM = sizeof(S) == 16;
    constexpr int NWARP = tr_threads<S>() / 32;
    extern __shared__ double tr_sm[];
    __shared__ int s_perm[NWARP][CO_MAX_K];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    S *W = reinterpret_cast<S *>(tr_sm) + warp * TR_WARP_D;
    S *sums = W;
    int *perm = s_perm[warp];
    const double eps = sizeof(T) == 8 ? DBL_EPSILON : (double)FLT_EPSILON;
    for (int m = blockIdx.x * NWARP + warp; m < p.M; m += gridDim.x * NWARP) {
        const uint8_t mode = p.imode[m];
        if (!(mode & IM_TR) || ((mode & IM_TR_DD) != 0) != DDM) continue;
        int st = p.status[m];
        if (st != ST_RUNNING || !p.pending[m]) continue;
        const TreeDesc dsc = p.desc[m];
        const int K = dsc.K, P = nblock_size(K), tri = K * (K + 1) / 2;
        for (int e = lane; e < P; e += 32) {
            if constexpr (DDM) {
                sums[e] = S(p.ddg[2 * (dsc.q_off + e)], p.ddg[2 * (dsc.q_off + e) + 1]);
            } else {
                const T *src = p.partials + dsc.p_off + e;
                T s = T(0);
                for (int ch = 0; ch < dsc.n_chunks; ++ch) s += src[(int64_t)ch * P];
                sums[e] = (double)s;
            }
        }
        __syncwarp();
        double *trs = p.tr + (int64_t)m * TR_FIELDS;
        const double ssq = to_double(sums[P - 1]);   // |f_try|^2
        const T ltry = T(0.5) * (T)ssq;
        const int ne = p.n_eval[m];                  // evaluations before this one
        const bool initial = ne == 0;
        __syncwarp();
        if (lane == 0) {
            p.pending[m] = 0;
            p.n_eval[m] = ne + 1;
        }
        double delta = trs[TR_DELTA], par = trs[TR_PAR], fnorm = trs[TR_FNORM];
        double xnorm = trs[TR_XNORM], pnorm = trs[TR_PNORM], gnorm = trs[TR_GNORM];
        int outer = p.outer[m];
        bool accept = false, done = false;
        double d = lane < K ? p.diag[dsc.c_off + lane] : 1.0;
        if (initial) {
            if (lane == 0) { p.loss_init[m] = ltry; p.loss[m] = ltry; }
            if (K == 0) { st = STATUS_K0_SKIP; done = true; }
            else if (!isfinite(ssq)) { st = STATUS_FAIL_NAN; done = true; }
            else { accept = true; fnorm = sqrt(ssq); outer = 1; }
        } else {
            if (lane == 0) p.iters[m] += 1;
            const double fnorm1 = isfinite(ssq) ? sqrt(ssq) : INFINITY;
            // |J p|^2 = p^T A p with A = the accepted point's J^T J (packed lower in blk, or
            // blk_dd for double-double fits)
            const double pk = lane < K ? (double)p.delta[dsc.c_off + lane] : 0.0;
            S ap = S(0.0);
            for (int l = 0; l < K; ++l) {
                const double pl = __shfl_sync(0xffffffffu, pk, l);
                if (lane < K) {
                    const int hi = lane > l ? lane : l, lo = lane > l ? l : lane;
                    const int64_t e = dsc.q_off + hi * (hi + 1) / 2 + lo;
                    if constexpr (DDM) ap += S(p.blk_dd[2 * e], p.blk_dd[2 * e + 1]) * S(pl);
                    else ap += S((double)p.blk[e]) * S(pl);
                }
            }
            const double jp2 = fmax(to_double(wl_sum(S(pk) * ap)), 0.0);
            const double actred = (0.1 * fnorm1 < fnorm) ? 1.0 - (fnorm1 / fnorm) * (fnorm1 / fnorm) : -1.0;
            const double t1 = sqrt(jp2) / fnorm, t2 = sqrt(par) * pnorm / fnorm;
            const double prered = t1 * t1 + t2 * t2 / 0.5;
            const double dirder = -(t1 * t1 + t2 * t2);
            const double ratio = prered != 0.0 ? actred / prered : 0.0;
            if (ratio <= 0.25) {
                double temp = actred >= 0.0 ? 0.5 : 0.5 * dirder / (dirder + 0.5 * actred);
                if (0.1 * fnorm1 >= fnorm || temp < 0.1) temp = 0.1;
                delta = temp * fmin(delta, pnorm / 0.1);
                par = par / temp;
            } else if (par == 0.0 || ratio >= 0.75) {
                delta = pnorm / 0.5;
                par = 0.5 * par;
            }
            if (ratio >= 1e-4) {
                accept = true;
                fnorm = fnorm1;
                outer += 1;
                const double cn = lane < K ? d * (double)p.ctry[dsc.c_off + lane] : 0.0;
                xnorm = wl_norm(cn);
                if (lane < K) p.c[dsc.c_off + lane] = p.ctry[dsc.c_off + lane];
                if (lane == 0) p.loss[m] = ltry;
            }
            if (fabs(actred) <= p.ftol && prered <= p.ftol && 0.5 * ratio <= 1.0) done = true;
            if (delta <= p.xtol * xnorm) done = true;
            if (fabs(actred) <= eps && prered <= eps && 0.5 * ratio <= 1.0) done = true;
            if (delta <= eps * xnorm) done = true;
            if (done) {
                st = STATUS_CONVERGED;
            } else if (ne + 1 >= p.max_nfev) {     // evaluation budget (MINPACK maxfev)
                st = STATUS_MAXITER;
                done = true;
            }
        }
        __syncwarp();
        if (accept) {
            // the new point's J^T J, J^T f must be finite to take a step from it
            bool bad = false;
            for (int e = lane; e < P; e += 32) bad |= !isfinite(sums[e]);
            if (__any_sync(0xffffffffu, bad) && !done) {
                st = STATUS_FAIL_NAN;
                done = true;
            }
            for (int e = lane; e < P; e += 32) {
                p.blk[dsc.q_off + e] = (T)to_double(sums[e]);
                if constexpr (DDM) {
                    p.blk_dd[2 * (dsc.q_off + e)] = sums[e].hi;
                    p.blk_dd[2 * (dsc.q_off + e) + 1] = sums[e].lo;
                }
            }
        }
        __syncwarp();
        if (!done) {
            // current point's J^T J and J^T f, from the accepted block (written above by this
            // warp; the warp barrier orders those writes before these reads)
            __syncwarp();
            const TrA<T, S> A{p.blk + dsc.q_off, DDM ? p.blk_dd + 2 * dsc.q_off : nullptr};
            S g = S(0.0);
            if (lane < K) {
                if constexpr (DDM) g = S(p.blk_dd[2 * (dsc.q_off + tri + lane)],
                                         p.blk_dd[2 * (dsc.q_off + tri + lane) + 1]);
                else g = S((double)p.blk[dsc.q_off + tri + lane]);
            }
            if (accept) {
                // outer iteration: column norms, the scaling, the gradient test
                const double acn = lane < K ? sqrt(fmax(to_double(A(lane, lane)), 0.0)) : 0.0;
                if (outer == 1) {
                    d = (lane < K && acn != 0.0) ? acn : 1.0;
                    const double cn = lane < K ? d * (double)p.c[dsc.c_off + lane] : 0.0;
                    xnorm = wl_norm(cn);
                    delta = xnorm != 0.0 ? p.factor * xnorm : p.factor;
                }
                double gl = 0.0;
                if (fnorm != 0.0 && lane < K && acn != 0.0) gl = fabs(to_double(g) / fnorm) / acn;
                gnorm = wl_max(gl);
                if (gnorm <= p.gtol || gnorm <= eps) {
                    st = STATUS_CONVERGED;
                    done = true;
                }
                d = fmax(d, acn);
            }
            if (!done) {
                const double x = to_double(tr_lmpar(A, W, perm, K, lane, g, d, delta, par));
                pnorm = wl_norm(lane < K ? d * x : 0.0);
                if (outer == 1) delta = fmin(delta, pnorm);
                if (lane < K) {
                    const T xk = (T)x;
                    p.delta[dsc.c_off + lane] = xk;
                    p.ctry[dsc.c_off + lane] = p.c[dsc.c_off + lane] + xk;
                }
                if (lane == 0) p.pending[m] = 1;
            }
        }
        if (lane < K) p.diag[dsc.c_off + lane] = d;
        if (lane == 0) {
            trs[TR_DELTA] = delta; trs[TR_PAR] = par; trs[TR_FNORM] = fnorm;
            trs[TR_XNORM] = xnorm; trs[TR_PNORM] = pnorm; trs[TR_GNORM] = gnorm;
            p.outer[m] = outer;
            p.status[m] = st;
            if (st == ST_RUNNING) atomicAdd(p.n_running, 1);
        }
        __syncwarp();
    }
}

}  // namespace cusr

namespace cusr {

// Normal equations of the trust-region fits that take them in double-double (IM_TR_DD), from
// the pass's per-sample values (vals[fit][N]) and Jacobian (jac[fit][jac_kmax][N], fp64):
// ddg holds, per fit at its q_off, the packed (K+1) x (K+1) lower triangle of the Gram matrix
// of [g_0 .. g_{K-1}; r] as (hi, lo) pairs — J^T J, J^T r, sum r^2. r = f - y with the
// sentinel convention of the fused pass (a non-finite residual counts as RESIDUAL_SENTINEL
// and its Jacobian row as 0).
// One block per fit; samples are staged through shared memory in tiles of DDG_TILE, the next
// tile's loads in flight in registers while a tile is summed. Each
// Gram entry is taken by G = DDG_THREADS / P threads (P entries), thread g of an entry
// summing the tile's samples g, g + G, ...: within a tile by Dot2 (Ogita, Rump & Oishi 2005,
// "Accurate sum and dot product": TwoProduct by fma, TwoSum of the running sum, the error
// terms summed apart), the tile's pair then added to the thread's double-double total; the G
// totals of an entry are added in g order at the end. The order of every sum is fixed.
constexpr int DDG_THREADS = 256;
constexpr int DDG_TILE = 64;
constexpr int DDG_LD = DDG_TILE + 1;          // odd row stride: rows read at one column spread
constexpr int DDG_PER_THREAD = (nblock_size(CO_MAX_K) + DDG_THREADS - 1) / DDG_THREADS;
// tile elements a thread stages: (K + 1) rows x DDG_TILE samples over the block
constexpr int DDG_NV = ((CO_MAX_K + 1) * DDG_TILE + DDG_THREADS - 1) / DDG_THREADS;

__global__ void __launch_bounds__(DDG_THREADS)
dd_gram_kernel(const TreeDesc *desc, int M, const uint8_t *imode, const int32_t *status,
               const int32_t *pending, const double *vals, const double *jac, int jac_kmax,
               const float *ym, int N, double *ddg) {
    __shared__ double tile[(CO_MAX_K + 1) * DDG_LD];
    __shared__ DD red[DDG_THREADS];
    for (int m = blockIdx.x; m < M; m += gridDim.x) {
        if (!(imode[m] & IM_TR_DD) || status[m] != ST_RUNNING || !pending[m]) continue;
        const TreeDesc d = desc[m];
        const int K = d.K, P = nblock_size(K);
        const int G = P <= DDG_THREADS ? DDG_THREADS / P : 1;   // threads per entry
        int ei[DDG_PER_THREAD], el[DDG_PER_THREAD], eg[DDG_PER_THREAD];
        bool on[DDG_PER_THREAD];
        DD acc[DDG_PER_THREAD];
#pragma unroll
        for (int q = 0; q < DDG_PER_THREAD; ++q) {
            const int u = threadIdx.x + q * DDG_THREADS;
            on[q] = u < G * P;
            const int e = on[q] ? u % P : 0;
            eg[q] = on[q] ? u / P : 0;
            int i = 0;
            while ((i + 1) * (i + 2) / 2 <= e) ++i;
            ei[q] = i;
            el[q] = e - i * (i + 1) / 2;
            acc[q] = DD(0.0);
        }
        const double *vrow = vals + (int64_t)m * N;
        const float *yrow = ym + d.y_off;
        const double *jrow = jac + (int64_t)m * jac_kmax * N;
        const int n_el = (K + 1) * DDG_TILE;
        // the next tile's raw values in registers (loads in flight while a tile is summed):
        // element idx = row * DDG_TILE + j, row K the value f (with its target), rows < K J
        double nv[DDG_NV];
        float ny[DDG_NV];
        auto fetch = [&](int s0) {
#pragma unroll
            for (int q = 0; q < DDG_NV; ++q) {
                const int idx = threadIdx.x + q * DDG_THREADS;
                const int row = idx / DDG_TILE, s = s0 + idx - row * DDG_TILE;
                nv[q] = 0.0;
                ny[q] = 0.f;
                if (idx < n_el && s < N) {
                    if (row == K) {
                        nv[q] = vrow[s];
                        ny[q] = yrow[s];
                    } else {
                        nv[q] = jrow[(int64_t)row * N + s];
                    }
                }
            }
        };
        fetch(0);
        for (int s0 = 0; s0 < N; s0 += DDG_TILE) {
            __syncthreads();
#pragma unroll
            for (int q = 0; q < DDG_NV; ++q) {
                const int idx = threadIdx.x + q * DDG_THREADS;
                if (idx < n_el) {
                    const int row = idx / DDG_TILE, j = idx - row * DDG_TILE;
                    tile[row * DDG_LD + j] = row == K ? nv[q] - (double)ny[q] : nv[q];
                }
            }
            __syncthreads();
            // the sentinel convention: a non-finite residual counts as RESIDUAL_SENTINEL and
            // its sample's Jacobian row as 0 (samples past N stay 0)
            if (threadIdx.x < DDG_TILE && !::isfinite(tile[K * DDG_LD + threadIdx.x])) {
                tile[K * DDG_LD + threadIdx.x] = RESIDUAL_SENTINEL;
                for (int row = 0; row < K; ++row) tile[row * DDG_LD + threadIdx.x] = 0.0;
            }
            if (s0 + DDG_TILE < N) fetch(s0 + DDG_TILE);
            __syncthreads();
#pragma unroll
            for (int q = 0; q < DDG_PER_THREAD; ++q) {
                if (on[q]) {
                    const double *a = tile + ei[q] * DDG_LD, *b = tile + el[q] * DDG_LD;
                    double ps = 0.0, err = 0.0;          // Dot2 over this thread's samples
                    for (int j = eg[q]; j < DDG_TILE; j += G) {
                        const double h = a[j] * b[j];
                        const double rr = fma(a[j], b[j], -h);
                        const double t = ps + h;
                        const double bb = t - ps;
                        err += ((ps - (t - bb)) + (h - bb)) + rr;
                        ps = t;
                    }
                    acc[q] += dd_two_sum(ps, err);
                }
            }
        }
        // the G partial totals of each entry, added in thread order
#pragma unroll
        for (int q = 0; q < DDG_PER_THREAD; ++q) {
            const int u = threadIdx.x + q * DDG_THREADS;
            if (G == 1) {
                if (on[q]) {
                    ddg[2 * (d.q_off + u)] = acc[q].hi;
                    ddg[2 * (d.q_off + u) + 1] = acc[q].lo;
                }
            } else if (q == 0) {
                __syncthreads();
                red[threadIdx.x] = on[0] ? acc[0] : DD(0.0);
                __syncthreads();
                if (threadIdx.x < P) {
                    DD t = red[threadIdx.x];
                    for (int g = 1; g < G; ++g) t += red[g * P + threadIdx.x];
                    ddg[2 * (d.q_off + threadIdx.x)] = t.hi;
                    ddg[2 * (d.q_off + threadIdx.x) + 1] = t.lo;
                }
            }
        }
    }
}

}  // namespace cusr
