// starts.cuh — the start axis: S fits per tree, fit i = tree * S + s, all in one batch.
//
// The programs are compiled once per tree; every fit of a tree shares them (its TreeDesc
// points at the same code), with constants, state and partial sums of its own. Start 0 is the
// tree's c_init; start s >= 1 is, cycling over four kinds, a log-normal scaling of c_init
// (c * exp(z1 / 2) + z2 / 20), a shift (c + (|c| + 1) z1 / 2), a fresh N(0, 1) draw and a fresh
// N(0, 9) draw, with z1, z2 standard normal numbers from a counter-based generator (SplitMix64
// mixing of (seed, tree, start, constant), Steele, Lea & Flood 2014; Box-Muller transform), so
// the points depend only on the seed and the position, never on the launch.
// Waves: starts s < wave1 run first; when they have all finished, a tree whose fits agree (two
// or more within agree_tol of the lowest loss) retires its other starts unrun, any other tree
// starts them. At the end every tree reports its start with the lowest final loss.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "lm_kernels.cuh"
#include "tr_step.cuh"

namespace cusr {

constexpr int32_t ST_WAITING = -2;   // a later-wave start that has not begun
constexpr int32_t ST_RETIRED = -3;   // a later-wave start its tree did not need

__host__ __device__ inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// standard normal number j (0, 1) of constant k of start s of tree m
__device__ inline double start_normal(uint64_t seed, int64_t m, int s, int k, int j) {
    uint64_t h = mix64(seed ^ mix64((uint64_t)m));
    h = mix64(h ^ (((uint64_t)(uint32_t)s << 32) | (uint64_t)(uint32_t)(2 * k + j)));
    const uint64_t h2 = mix64(h);
    const double u1 = ((double)(h >> 11) + 0.5) * 0x1.0p-53;   // (0, 1)
    const double u2 = (double)(h2 >> 11) * 0x1.0p-53;          // [0, 1)
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

template <typename T>
struct StartsParams {
    const TreeDesc *desc;      // per fit
    const int32_t *tree_coff;  // per tree: offset of its constants in the caller's c_init
    const float *c_tree;       // the caller's c_init (per tree)
    int M_fit, S, wave1, tr_starts;
    int damp_alternate;        // reference fits alternate the floored damping on every solve
    int tr_dd;                 // trust-region fits take double-double normal equations
    uint64_t seed;
    T lam0;
    float *c_start;            // per fit constant: the start point (the audit's c_init)
    T *c, *ctry, *lam;
    int32_t *status, *iters, *pending, *n_eval, *outer;
    uint8_t *imode;
    double *tr, *diag;
};

template <typename T>
__global__ void init_starts_kernel(const StartsParams<T> p) {
    const int64_t gs = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.M_fit; i += gs) {
        const int64_t m = i / p.S;
        const int s = (int)(i - m * p.S);
        const TreeDesc d = p.desc[i];
        const float *c0 = p.c_tree + p.tree_coff[m];
        for (int k = 0; k < d.K; ++k) {
            double v = c0[k];
            if (s > 0) {
                const double z1 = start_normal(p.seed, m, s, k, 0);
                switch ((s - 1) % 4) {
                    case 0: v = v * exp(0.5 * z1) + 0.05 * start_normal(p.seed, m, s, k, 1); break;
                    case 1: v = v + 0.5 * (fabs(v) + 1.0) * z1; break;
                    case 2: v = z1; break;
                    default: v = 3.0 * z1; break;
                }
            }
            const float vf = (float)v;
            p.c_start[d.c_off + k] = vf;
            p.c[d.c_off + k] = (T)vf;
            p.ctry[d.c_off + k] = (T)vf;
            p.diag[d.c_off + k] = 1.0;
        }
        uint8_t mode = 0;
        if (s < p.tr_starts) mode = IM_TR | IM_SENTINEL | (p.tr_dd ? IM_TR_DD : 0);
        else if (p.damp_alternate && ((s - p.tr_starts) & 1)) mode = IM_DAMP_ALWAYS;
        p.imode[i] = mode;
        const bool first = p.wave1 <= 0 || s < p.wave1;
        p.status[i] = first ? ST_RUNNING : ST_WAITING;
        p.pending[i] = first ? 1 : 0;
        p.lam[i] = p.lam0;
        p.iters[i] = 0;
        p.n_eval[i] = 0;
        p.outer[i] = 0;
        for (int f = 0; f < TR_FIELDS; ++f) p.tr[i * TR_FIELDS + f] = 0.0;
    }
}

// After each step: trees whose first wave has finished retire or start their later starts.
template <typename T>
__global__ void waves_kernel(int M, int S, int wave1, double agree_tol, const T *loss,
                             int32_t *status, int32_t *pending, uint8_t *resolved,
                             int *n_running, int *n_retired) {
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        if (resolved[m]) continue;
        const int64_t b = (int64_t)m * S;
        bool busy = false;
        double best = INFINITY;
        for (int s = 0; s < wave1; ++s) {
            const int32_t st = status[b + s];
            busy |= st == ST_RUNNING;
            const double l = (double)loss[b + s];
            if ((st == STATUS_CONVERGED || st == STATUS_MAXITER) && l < best) best = l;
        }
        if (busy) continue;
        int agree = 0;
        for (int s = 0; s < wave1; ++s) {
            const int32_t st = status[b + s];
            const double l = (double)loss[b + s];
            if ((st == STATUS_CONVERGED || st == STATUS_MAXITER) && l <= best + agree_tol * fabs(best))
                ++agree;
        }
        // K = 0 trees and trees no fit of which finished cleanly have nothing to gain
        const bool retire = agree >= 2 || status[b] == STATUS_K0_SKIP || !isfinite(best);
        int started = 0;
        for (int s = wave1; s < S; ++s) {
            if (retire) {
                status[b + s] = ST_RETIRED;
            } else {
                status[b + s] = ST_RUNNING;
                pending[b + s] = 1;
                ++started;
            }
        }
        resolved[m] = 1;
        if (retire) atomicAdd(n_retired, 1);
        if (started) atomicAdd(n_running, started);
    }
}

// Per tree, the start with the lowest final loss: the fp64 audit loss when the call audited
// (l64 = [final | at start] per fit), else the fit's own loss. Ties: the lower start index.
template <typename T>
__global__ void select_best_kernel(const TreeDesc *desc, const int32_t *tree_coff, int M, int S,
                                   const T *loss, const T *loss_init, const double *l64,
                                   const int32_t *status, const int32_t *iters,
                                   const int32_t *n_eval, const T *c, T *out_c,
                                   int32_t *out_status, T *out_li, T *out_lf, int32_t *out_iters,
                                   int32_t *out_start) {
    const int64_t Mf = (int64_t)M * S;
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const int64_t b = (int64_t)m * S;
        int best_s = 0;
        double best = INFINITY;
        for (int s = 0; s < S; ++s) {
            const int64_t i = b + s;
            if (n_eval[i] == 0) continue;       // waiting / retired: never evaluated
            double key = (double)loss[i];
            if (l64) {
                const double lf = l64[i], li = l64[Mf + i];
                key = (!isfinite(lf) || (isfinite(li) && lf > li)) ? li : lf;
            }
            if (isfinite(key) && key < best) { best = key; best_s = s; }
        }
        const int64_t i = b + best_s;
        const TreeDesc d = desc[i];
        for (int k = 0; k < d.K; ++k) out_c[tree_coff[m] + k] = c[d.c_off + k];
        const int32_t st = status[i];
        out_status[m] = (st == ST_RUNNING || st == ST_WAITING || st == ST_RETIRED) ? STATUS_MAXITER : st;
        out_li[m] = loss_init[b];
        out_lf[m] = loss[i];
        out_iters[m] = iters[i];
        out_start[m] = best_s;
    }
}

}  // namespace cusr
