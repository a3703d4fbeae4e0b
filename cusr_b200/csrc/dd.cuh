// dd.cuh — double-double arithmetic (a value is hi + lo, |lo| <= ulp(hi) / 2, about 106
// significant bits) for the trust-region step's normal equations (dd_gram_kernel and
// lm_tr_step_kernel_dd in tr_step.cuh).
//
// The algorithms are the published error-free transformations: TwoSum (Knuth, TAOCP vol. 2,
// 4.2.2), FastTwoSum (Dekker 1971), TwoProduct with a fused multiply-add, and the
// double-double addition, multiplication, division and square root built on them (Dekker
// 1971; Hida, Li & Bailey 2001, "Algorithms for quad-double precision floating point
// arithmetic"). Only IEEE add / multiply / fma / divide / sqrt of doubles are used.
//
// Why: on trees whose Jacobian is rank-deficient to about machine precision, J^T J formed in
// fp64 loses the small singular directions (its rounding is eps |J|^2, their weight
// sigma^2 << eps |J|^2), so the trust-region step takes the basic solution where MINPACK's
// QR of J keeps them; with J^T J accumulated and factored in double-double the step keeps
// them too (a 24-digit restatement already reproduces MINPACK's fits on such trees).
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include "program.h"

namespace cusr {

// the double overloads stay visible next to the DD ones declared below
using ::fabs;
using ::isfinite;
using ::sqrt;

struct DD {
    double hi, lo;
    DD() = default;
    __host__ __device__ constexpr DD(double a) : hi(a), lo(0.0) {}
    __host__ __device__ constexpr DD(double h, double l) : hi(h), lo(l) {}
};

__device__ __forceinline__ DD dd_two_sum(double a, double b) {
    const double s = a + b;
    const double bb = s - a;
    return DD(s, (a - (s - bb)) + (b - bb));
}
__device__ __forceinline__ DD dd_fast_two_sum(double a, double b) {   // |a| >= |b|
    const double s = a + b;
    return DD(s, b - (s - a));
}
__device__ __forceinline__ DD dd_two_prod(double a, double b) {
    const double p = a * b;
    return DD(p, fma(a, b, -p));
}

__device__ __forceinline__ DD operator+(DD a, DD b) {
    DD s = dd_two_sum(a.hi, b.hi);
    const DD t = dd_two_sum(a.lo, b.lo);
    s.lo += t.hi;
    s = dd_fast_two_sum(s.hi, s.lo);
    s.lo += t.lo;
    return dd_fast_two_sum(s.hi, s.lo);
}
__device__ __forceinline__ DD operator-(DD a) { return DD(-a.hi, -a.lo); }
__device__ __forceinline__ DD operator-(DD a, DD b) { return a + (-b); }
__device__ __forceinline__ DD operator*(DD a, DD b) {
    DD p = dd_two_prod(a.hi, b.hi);
    p.lo += a.hi * b.lo + a.lo * b.hi;
    return dd_fast_two_sum(p.hi, p.lo);
}
__device__ __forceinline__ DD operator/(DD a, DD b) {
    const double q1 = a.hi / b.hi;
    DD r = a - b * DD(q1);
    const double q2 = r.hi / b.hi;
    r = r - b * DD(q2);
    const double q3 = r.hi / b.hi;
    return dd_fast_two_sum(q1, q2) + DD(q3);
}
__device__ __forceinline__ DD &operator+=(DD &a, DD b) { return a = a + b; }
__device__ __forceinline__ DD &operator-=(DD &a, DD b) { return a = a - b; }
__device__ __forceinline__ DD &operator*=(DD &a, DD b) { return a = a * b; }
__device__ __forceinline__ DD &operator/=(DD &a, DD b) { return a = a / b; }

__device__ __forceinline__ bool operator<(DD a, DD b) { return a.hi < b.hi || (a.hi == b.hi && a.lo < b.lo); }
__device__ __forceinline__ bool operator>(DD a, DD b) { return b < a; }
__device__ __forceinline__ bool operator<=(DD a, DD b) { return !(b < a) && a.hi == a.hi && b.hi == b.hi; }
__device__ __forceinline__ bool operator>=(DD a, DD b) { return b <= a; }
__device__ __forceinline__ bool operator==(DD a, DD b) { return a.hi == b.hi && a.lo == b.lo; }
__device__ __forceinline__ bool operator!=(DD a, DD b) { return !(a == b); }

// square root: the double root refined by one Newton step in double-double
__device__ __forceinline__ DD sqrt(DD a) {
    if (!(a.hi > 0.0)) return DD(::sqrt(a.hi));       // 0, negative (NaN) or NaN
    const double q = ::sqrt(a.hi);
    const DD r = a - dd_two_prod(q, q);
    return dd_fast_two_sum(q, r.hi / (2.0 * q));
}
__device__ __forceinline__ DD fabs(DD a) { return a.hi < 0.0 ? -a : a; }
__device__ __forceinline__ bool isfinite(DD a) { return ::isfinite(a.hi); }
__device__ __forceinline__ double to_double(DD a) { return a.hi + a.lo; }
__device__ __forceinline__ double to_double(double a) { return a; }

__device__ __forceinline__ DD shfl(DD v, int src) {
    return DD(__shfl_sync(0xffffffffu, v.hi, src), __shfl_sync(0xffffffffu, v.lo, src));
}
__device__ __forceinline__ DD shfl_xor(DD v, int mask) {
    return DD(__shfl_xor_sync(0xffffffffu, v.hi, mask), __shfl_xor_sync(0xffffffffu, v.lo, mask));
}
__device__ __forceinline__ double shfl(double v, int src) { return __shfl_sync(0xffffffffu, v, src); }
__device__ __forceinline__ double shfl_xor(double v, int mask) {
    return __shfl_xor_sync(0xffffffffu, v, mask);
}

}  // namespace cusr
