// ops.h — value and local partial derivatives of every operator, shared by the device
// interpreter and the host-side program checker so both compute the same thing.
//
// Value semantics follow the reference's CUDA interpreter and numpy oracle
// (cusr/kernel/lm_core.cuh:58-106, cusr/benchmark/interp.py:32-49); derivative rules follow
// its reverse-mode interpreter (cusr/kernel/revad_interp.cuh:86-131):
//   SIN d=cos a, COS d=-sin a, TAN d=1+r^2, SINH d=cosh a, COSH d=sinh a, TANH d=1-r^2,
//   LOG d=1/a, EXP d=r, INV d=-r^2, NEG d=-1, ABS d=sign0(a), SQRT d=1/(2r);
//   ADD (1,1), SUB (1,-1), MUL (b,a), DIV (1/b, -o/b), POW (b*a^(b-1), o*log a),
//   MAX/MIN select (ties to the left operand), comparisons (0,0).
// The LOOSE_* operators of the numpy oracle (log|a|, sqrt|a|, |a|^b, 1/a, a/b) are
// implemented natively (the reference CUDA kernel maps them to 0); their derivatives are
// those of the same formulas. Unknown operator ids evaluate to 0 with zero derivative,
// as in the reference kernel. MAX/MIN propagate NaN like numpy's maximum/minimum.
#pragma once
#include <math.h>
#include "program.h"

#define CUSR_HD __host__ __device__ __forceinline__

namespace cusr {

#if defined(__CUDA_ARCH__) && defined(CUSR_SFU)
// The default fp32 arithmetic (the translation unit built with CUSR_SFU): the special-function
// unit (MUFU) where one Newton step or an exact argument split brings its result to about one
// ulp, and our own argument reduction and polynomials for sin / cos; IEEE library calls remain
// for log and for the rare arguments outside the reduced ranges. Accuracy (measured against
// fp64): sin / cos within 3 * 2^-24 relative for |x| <= 1e5 (Cody & Waite 1980 reduction by
// pi/2 with a three-part constant, degree-7 / degree-8 polynomials on [-pi/4, pi/4] fitted by
// Lawson-reweighted least squares on Chebyshev nodes); exp from 2^f on |f| <= 1/2 after an
// exact hi/lo split of x * log2(e); reciprocal one Newton-Raphson step on the hardware
// approximation; square root the hardware approximation.
namespace sfu {
__device__ __forceinline__ float bits(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ float rcp_hw(float b) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(b));
    return r;
}
__device__ __forceinline__ float ex2_hw(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float sqrt_hw(float x) {
    float r;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// 1 / b: a Newton-Raphson step r + r (1 - b r) on the hardware estimate; b = 0, +-inf (where
// the residual is NaN) keep the estimate, which is then exact (+-inf, +-0)
__device__ __forceinline__ float rcp(float b) {
    const float r = rcp_hw(b);
    const float e = fmaf(-b, r, 1.0f);
    const float r1 = fmaf(r, e, r);
    return e == e ? r1 : r;
}
__device__ __noinline__ void sincos_wide(float x, float *s, float *c) { ::sincosf(x, s, c); }
__device__ __noinline__ float exp_wide(float x) { return ::expf(x); }
__device__ __forceinline__ void sincos(float x, float *s, float *c) {
    if (!(fabsf(x) <= 1e5f)) {     // large or non-finite arguments: the library's reduction
        sincos_wide(x, s, c);
        return;
    }
    const float k = rintf(x * bits(0x3f22f983u));                 // x * 2/pi
    float r = fmaf(-k, bits(0x3fc90fdbu), x);                      // pi/2 = P1 + P2 + P3
    r = fmaf(-k, bits(0xb33bbd2eu), r);
    r = fmaf(-k, bits(0xa6f72cedu), r);
    const float r2 = r * r;
    float ps = fmaf(r2, bits(0xb94ca1f0u), bits(0x3c08839du));
    ps = fmaf(r2, ps, bits(0xbe2aaaa3u));
    const float sr = fmaf(r2 * r, ps, r);                          // sin r
    float pc = fmaf(r2, bits(0x37cc8b50u), bits(0xbab603f9u));
    pc = fmaf(r2, pc, bits(0x3d2aaa9eu));
    pc = fmaf(r2, pc, -0.5f);
    const float cr = fmaf(r2, pc, 1.0f);                           // cos r
    const int q = (int)k & 3;
    const float a = (q & 1) ? cr : sr, b = (q & 1) ? sr : cr;
    *s = (q & 2) ? -a : a;
    *c = ((q + 1) & 2) ? -b : b;
}
__device__ __forceinline__ float exp(float x) {
    if (!(fabsf(x) <= 87.0f)) return exp_wide(x);                 // overflow / underflow
    const float t = x * bits(0x3fb8aa3bu);                         // x log2(e), high part
    float lo = fmaf(x, bits(0x3fb8aa3bu), -t);                     // its exact rounding error
    lo = fmaf(x, bits(0x32a57060u), lo);                           // + x * (log2(e) - high)
    const float n = rintf(t);
    const float e = ex2_hw((t - n) + lo);                          // 2^f, |f| <= 1/2 + tiny
    return __int_as_float(__float_as_int(e) + ((int)n << 23));     // * 2^n, n in [-126, 126]
}
}  // namespace sfu
#endif

template <typename T> struct Mth;
template <> struct Mth<float> {
    static CUSR_HD float sin(float a) { return ::sinf(a); }
    static CUSR_HD float cos(float a) { return ::cosf(a); }
    static CUSR_HD void sincos(float a, float *s, float *c) {
#if defined(__CUDA_ARCH__) && defined(CUSR_SFU)
        sfu::sincos(a, s, c);
#elif defined(__CUDA_ARCH__)
        ::sincosf(a, s, c);
#else
        *s = ::sinf(a); *c = ::cosf(a);
#endif
    }
    static CUSR_HD float tan(float a) { return ::tanf(a); }
    static CUSR_HD float sinh(float a) { return ::sinhf(a); }
    static CUSR_HD float cosh(float a) { return ::coshf(a); }
    static CUSR_HD float tanh(float a) { return ::tanhf(a); }
    static CUSR_HD float log(float a) { return ::logf(a); }
#if defined(__CUDA_ARCH__) && defined(CUSR_SFU)
    static CUSR_HD float exp(float a) { return sfu::exp(a); }
    static CUSR_HD float sqrt(float a) { return sfu::sqrt_hw(a); }
#else
    static CUSR_HD float exp(float a) { return ::expf(a); }
    static CUSR_HD float sqrt(float a) { return ::sqrtf(a); }
#endif
    static CUSR_HD float pow(float a, float b) { return ::powf(a, b); }
    static CUSR_HD float fabs(float a) { return ::fabsf(a); }
    static CUSR_HD float copysign(float a, float b) { return ::copysignf(a, b); }
    // correctly rounded reciprocal: the same value as 1.0f / a, without a general division;
    // under --use_fast_math the reference's 1.0f / a is the approximate division, kept here
    static CUSR_HD float rcp(float a) {
#if defined(__CUDA_ARCH__) && defined(__USE_FAST_MATH__)
        return 1.0f / a;
#elif defined(__CUDA_ARCH__) && defined(CUSR_SFU)
        return sfu::rcp(a);
#elif defined(__CUDA_ARCH__)
        return __frcp_rn(a);
#else
        return 1.0f / a;
#endif
    }
    static CUSR_HD bool finite(float a) { return isfinite(a); }
    // a / b given r = rcp(b): IEEE division, or a * r in the SFU build (within 1.5 ulp)
    static CUSR_HD float quot(float a, float b, float r) {
#if defined(__CUDA_ARCH__) && defined(CUSR_SFU)
        (void)b;
        return a * r;
#else
        (void)r;
        return a / b;
#endif
    }
};
template <> struct Mth<double> {
    static CUSR_HD double sin(double a) { return ::sin(a); }
    static CUSR_HD double cos(double a) { return ::cos(a); }
    static CUSR_HD void sincos(double a, double *s, double *c) {
#ifdef __CUDA_ARCH__
        ::sincos(a, s, c);
#else
        *s = ::sin(a); *c = ::cos(a);
#endif
    }
    static CUSR_HD double tan(double a) { return ::tan(a); }
    static CUSR_HD double sinh(double a) { return ::sinh(a); }
    static CUSR_HD double cosh(double a) { return ::cosh(a); }
    static CUSR_HD double tanh(double a) { return ::tanh(a); }
    static CUSR_HD double log(double a) { return ::log(a); }
    static CUSR_HD double exp(double a) { return ::exp(a); }
    static CUSR_HD double sqrt(double a) { return ::sqrt(a); }
    static CUSR_HD double pow(double a, double b) { return ::pow(a, b); }
    static CUSR_HD double fabs(double a) { return ::fabs(a); }
    static CUSR_HD double copysign(double a, double b) { return ::copysign(a, b); }
    static CUSR_HD double rcp(double a) {
#ifdef __CUDA_ARCH__
        return __drcp_rn(a);
#else
        return 1.0 / a;
#endif
    }
    static CUSR_HD bool finite(double a) { return isfinite(a); }
    static CUSR_HD double quot(double a, double b, double) { return a / b; }
};

template <typename T> CUSR_HD T sign0(T a) {
    return a > T(0) ? T(1) : (a < T(0) ? T(-1) : T(0));
}

// reverse-mode edge product with exact-zero annihilation (revad_interp.cuh:45-47): a zero
// adjoint or a zero local partial contributes 0, never 0*inf = NaN.
template <typename T> CUSR_HD T safe_mul(T a, T b) {
    return (a == T(0) || b == T(0)) ? T(0) : a * b;
}

template <typename T> CUSR_HD void unary_op(uint32_t op, T a, T &r, T &d);
template <typename T> CUSR_HD void binary_op(uint32_t op, T a, T b, T &o, T &da, T &db);

#if defined(__CUDA_ARCH__)
// operators outside the common grammar run out of line, keeping the interpreter's hot code
// small; both helpers are the same formulas as below
template <typename T> __device__ __noinline__ void unary_rare(uint32_t op, T a, T &r, T &d);
template <typename T> __device__ __noinline__ void binary_rare(uint32_t op, T a, T b, T &o, T &da, T &db);
#define CUSR_IS_RARE_UN(op) ((op) == OP_TAN || (op) == OP_SINH || (op) == OP_COSH || (op) == OP_TANH)
#define CUSR_IS_RARE_BIN(op) ((op) == OP_POW || (op) == OP_POWABS)
#endif

// Unary operator: r = f(a), d = f'(a).
template <typename T> CUSR_HD void unary_op(uint32_t op, T a, T &r, T &d) {
    using M = Mth<T>;
#if defined(__CUDA_ARCH__)
    if (CUSR_IS_RARE_UN(op)) { unary_rare<T>(op, a, r, d); return; }
#endif
    switch (op) {
        case OP_SIN: { T s, c; M::sincos(a, &s, &c); r = s; d = c; break; }
        case OP_COS: { T s, c; M::sincos(a, &s, &c); r = c; d = -s; break; }
        case OP_TAN: r = M::tan(a); d = T(1) + r * r; break;
        case OP_SINH: r = M::sinh(a); d = M::cosh(a); break;
        case OP_COSH: r = M::cosh(a); d = M::sinh(a); break;
        case OP_TANH: r = M::tanh(a); d = T(1) - r * r; break;
        case OP_LOG: r = M::log(a); d = M::rcp(a); break;
        case OP_LOGABS: r = M::log(M::fabs(a)); d = M::rcp(a); break;
        case OP_EXP: r = M::exp(a); d = r; break;
        case OP_INV: r = M::rcp(a); d = -r * r; break;
        case OP_NEG: r = -a; d = T(-1); break;
        case OP_ABS: r = M::fabs(a); d = sign0(a); break;
        case OP_SQRT: r = M::sqrt(a); d = M::rcp(T(2) * r); break;
        case OP_SQRTABS: r = M::sqrt(M::fabs(a)); d = M::copysign(M::rcp(T(2) * r), a); break;
        default: r = T(0); d = T(0); break;
    }
}

// Binary operator: o = a OP b (a = left operand), da = do/da, db = do/db.
template <typename T> CUSR_HD void binary_op(uint32_t op, T a, T b, T &o, T &da, T &db) {
    using M = Mth<T>;
#if defined(__CUDA_ARCH__)
    if (CUSR_IS_RARE_BIN(op)) { binary_rare<T>(op, a, b, o, da, db); return; }
#endif
    switch (op) {
        case OP_ADD: o = a + b; da = T(1); db = T(1); break;
        case OP_SUB: o = a - b; da = T(1); db = T(-1); break;
        case OP_MUL: o = a * b; da = b; db = a; break;
        case OP_DIV: da = M::rcp(b); o = M::quot(a, b, da); db = -o * da; break;
        case OP_POW: o = M::pow(a, b); da = b * M::pow(a, b - T(1)); db = o * M::log(a); break;
        case OP_POWABS: {
            T aa = M::fabs(a);
            o = M::pow(aa, b);
            da = b * M::pow(aa, b - T(1)) * sign0(a);
            db = o * M::log(aa);
            break;
        }
        case OP_MAX:
            o = (a != a || b != b) ? a + b : (a >= b ? a : b);
            da = (a >= b) ? T(1) : T(0); db = T(1) - da; break;
        case OP_MIN:
            o = (a != a || b != b) ? a + b : (a <= b ? a : b);
            da = (a <= b) ? T(1) : T(0); db = T(1) - da; break;
        case OP_LT: o = (a < b) ? T(1) : T(0); da = T(0); db = T(0); break;
        case OP_GT: o = (a > b) ? T(1) : T(0); da = T(0); db = T(0); break;
        case OP_LE: o = (a <= b) ? T(1) : T(0); da = T(0); db = T(0); break;
        case OP_GE: o = (a >= b) ? T(1) : T(0); da = T(0); db = T(0); break;
        default: o = T(0); da = T(0); db = T(0); break;
    }
}

#if defined(__CUDA_ARCH__)
template <typename T> __device__ __noinline__ void unary_rare(uint32_t op, T a, T &r, T &d) {
    using M = Mth<T>;
    switch (op) {
        case OP_TAN: r = M::tan(a); d = T(1) + r * r; break;
        case OP_SINH: r = M::sinh(a); d = M::cosh(a); break;
        case OP_COSH: r = M::cosh(a); d = M::sinh(a); break;
        default: r = M::tanh(a); d = T(1) - r * r; break;
    }
}
template <typename T> __device__ __noinline__ void binary_rare(uint32_t op, T a, T b, T &o, T &da, T &db) {
    using M = Mth<T>;
    if (op == OP_POW) {
        o = M::pow(a, b); da = b * M::pow(a, b - T(1)); db = o * M::log(a);
    } else {
        T aa = M::fabs(a);
        o = M::pow(aa, b);
        da = b * M::pow(aa, b - T(1)) * sign0(a);
        db = o * M::log(aa);
    }
}
#endif

// Tape slots an instruction writes in the forward sweep (read back in the reverse sweep).
//   unary                      : d            (NEG, UZERO: none)
//   MUL  VAR / CONST / POP     : - / [ds] / [dt, ds]   (dt of VAR/CONST is the operand)
//   DIV, POW, POWABS           : [dt] (+ [ds] for CONST / POP)
//   MAX, MIN                   : [dt]   (ds = 1 - dt)
//   ADD, SUB, comparisons, zero: none
CUSR_HD int tape_slots(uint32_t op, uint32_t mode) {
    if (op == OP_LOAD) return 0;
    if (op < OP_ADD) return (op == OP_NEG || op == OP_UZERO) ? 0 : 1;
    switch (op) {
        case OP_MUL: return mode == M_VAR ? 0 : (mode == M_CONST ? 1 : 2);
        case OP_DIV: case OP_POW: case OP_POWABS: return mode == M_VAR ? 1 : 2;
        case OP_MAX: case OP_MIN: return 1;
        default: return 0;
    }
}

}  // namespace cusr
