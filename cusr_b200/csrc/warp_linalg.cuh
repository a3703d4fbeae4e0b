// warp_linalg.cuh — dense K x K (K <= 32) linear algebra by one warp, for the per-fit step
// kernels: lane i owns row i of a matrix in shared memory (row stride WL_LD doubles, odd, so
// that a column read by the 32 lanes touches distinct banks), vectors are lane-distributed
// (lane i holds element i, lanes >= K hold 0).
#pragma once
#include <cuda_runtime.h>
#include "program.h"

namespace cusr {

constexpr int WL_LD = CO_MAX_K + 1;   // padded row stride (doubles)

__device__ __forceinline__ double wl_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double wl_max(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Euclidean norm of a lane-distributed vector (the lanes >= K hold 0)
__device__ __forceinline__ double wl_norm(double v) { return sqrt(wl_sum(v * v)); }

// W (rows 0..K-1 owned by lanes) = L L^T in place (lower triangle), unpivoted. false if a
// pivot is not positive (the test reads shared memory every lane sees: warp-uniform).
__device__ bool wl_chol(double *W, int K, int lane) {
    for (int j = 0; j < K; ++j) {
        __syncwarp();
        const double djj = W[j * WL_LD + j];
        if (!(djj > 0.0)) return false;
        const double ljj = sqrt(djj);
        __syncwarp();
        if (lane > j && lane < K) W[lane * WL_LD + j] /= ljj;
        if (lane == j) W[j * WL_LD + j] = ljj;
        __syncwarp();
        if (lane > j && lane < K) {
            const double lij = W[lane * WL_LD + j];
            for (int k = j + 1; k <= lane; ++k) W[lane * WL_LD + k] -= lij * W[k * WL_LD + j];
        }
    }
    __syncwarp();
    return true;
}

// solve L y = b (lane i holds b_i, returns y_i), L lower in W
__device__ double wl_fsub(const double *W, int K, int lane, double b) {
    double y = 0.0;
    for (int k = 0; k < K; ++k) {
        double yk = 0.0;
        if (lane == k) yk = b / W[k * WL_LD + k];
        yk = __shfl_sync(0xffffffffu, yk, k);
        if (lane == k) y = yk;
        if (lane > k && lane < K) b -= W[lane * WL_LD + k] * yk;
    }
    return y;
}
// solve L^T x = y (lane i holds y_i, returns x_i)
__device__ double wl_bsub(const double *W, int K, int lane, double y) {
    double x = 0.0;
    for (int k = K - 1; k >= 0; --k) {
        double xk = 0.0;
        if (lane == k) xk = y / W[k * WL_LD + k];
        xk = __shfl_sync(0xffffffffu, xk, k);
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
