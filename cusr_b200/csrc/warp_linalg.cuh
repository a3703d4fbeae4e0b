// warp_linalg.cuh — dense K x K (K <= 32) linear algebra by one warp, for the per-fit step
// kernels: lane i owns row i of a matrix in shared memory (row stride WL_LD doubles, odd, so
// that a column read by the 32 lanes touches distinct banks), vectors are lane-distributed
// (lane i holds element i, lanes >= K hold 0). The scalar S is double or DD (double-double).
#pragma once
#include <cuda_runtime.h>
#include "../../include/cusr_co.h"
#include "program.h"
#include "dd.cuh"

namespace cusr {

constexpr int WL_LD = CO_MAX_K + 1;   // padded row stride (doubles)

__device__ __forceinline__ double smax(double a, double b) { return fmax(a, b); }
__device__ __forceinline__ DD smax(DD a, DD b) { return b > a ? b : a; }

template <typename S>
__device__ __forceinline__ S wl_sum(S v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_xor(v, o);
    return v;
}
template <typename S>
__device__ __forceinline__ S wl_max(S v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = smax(v, shfl_xor(v, o));
    return v;
}
// Euclidean norm of a lane-distributed vector (the lanes >= K hold 0), as a double
template <typename S>
__device__ __forceinline__ double wl_norm(S v) { return to_double(sqrt(wl_sum(v * v))); }

// W (rows 0..K-1 owned by lanes) = L L^T in place (lower triangle), unpivoted. false if a
// pivot is not positive (the test reads shared memory every lane sees: warp-uniform).
template <typename S>
__device__ bool wl_chol(S *W, int K, int lane) {
    for (int j = 0; j < K; ++j) {
        __syncwarp();
        const S djj = W[j * WL_LD + j];
        if (!(djj > S(0.0))) return false;
        const S ljj = sqrt(djj);
        __syncwarp();
        if (lane > j && lane < K) W[lane * WL_LD + j] /= ljj;
        if (lane == j) W[j * WL_LD + j] = ljj;
        __syncwarp();
        if (lane > j && lane < K) {
            const S lij = W[lane * WL_LD + j];
            for (int k = j + 1; k <= lane; ++k) W[lane * WL_LD + k] -= lij * W[k * WL_LD + j];
        }
    }
    __syncwarp();
    return true;
}

// solve L y = b (lane i holds b_i, returns y_i), L lower in W
template <typename S>
__device__ S wl_fsub(const S *W, int K, int lane, S b) {
    S y = S(0.0);
    for (int k = 0; k < K; ++k) {
        S yk = S(0.0);
        if (lane == k) yk = b / W[k * WL_LD + k];
        yk = shfl(yk, k);
        if (lane == k) y = yk;
        if (lane > k && lane < K) b -= W[lane * WL_LD + k] * yk;
    }
    return y;
}
// solve L^T x = y (lane i holds y_i, returns x_i)
template <typename S>
__device__ S wl_bsub(const S *W, int K, int lane, S y) {
    S x = S(0.0);
    for (int k = K - 1; k >= 0; --k) {
        S xk = S(0.0);
        if (lane == k) xk = y / W[k * WL_LD + k];
        xk = shfl(xk, k);
        if (lane == k) x = xk;
        if (lane < k) y -= W[k * WL_LD + lane] * xk;
    }
    return x;
}

template <typename T>
__device__ __forceinline__ T wl_sum_t(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Left-looking Cholesky of the lower triangle of W in place (lane i owns row i; the upper
// triangle is not read). Every element takes the operation order of the reference's serial
// solve (batch_lm_ad.cu:161-178): column j, l_jj = sqrt(a_jj - sum_k l_jk^2) and
// l_ij = (a_ij - sum_k l_ik l_jk) / l_jj, k ascending, so the factor is the serial one bit for
// bit, in O(K^2) warp steps instead of O(K^3) on one lane. false (warp-uniform) when a pivot
// is <= 0; a NaN pivot goes on, as in the reference.
__device__ bool wl_chol_left(double *W, int K, int lane) {
    for (int j = 0; j < K; ++j) {
        double t = 0.0;
        if (lane >= j && lane < K) {
            t = W[lane * WL_LD + j];
            for (int k = 0; k < j; ++k) t -= W[lane * WL_LD + k] * W[j * WL_LD + k];
        }
        const double s = __shfl_sync(0xffffffffu, t, j);
        if (s <= 0.0) return false;
        const double ljj = sqrt(s);
        if (lane == j) W[j * WL_LD + j] = ljj;
        else if (lane > j && lane < K) W[lane * WL_LD + j] = t / ljj;
        __syncwarp();
    }
    return true;
}

}  // namespace cusr
