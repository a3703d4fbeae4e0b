"""numpy restatement of the reference tree interpreter and its reverse-mode Jacobian.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Value semantics: cusr/benchmark/interp.py:15-74 (prefix bytecode evaluated right to left
with an (N,)-vector stack; a binary node pops its left operand first and computes
`left OP right`; LOOSE_* operators as in its UNARY/BINARY tables). Operator ids that the
reference CUDA kernel does not know evaluate to 0 there (cusr/kernel/lm_core.cuh:82,100);
this restatement does the same so such trees stay comparable.

Jacobian: reverse sweep of cusr/kernel/revad_interp.cuh:66-157 — per-node local partials
recorded in the forward pass, adjoints propagated root to leaves with the exact-zero
annihilating product `revad_safe_mul` (:45-47); constant leaves receive their adjoint.
"""
from __future__ import annotations

import numpy as np

NTYPE_VAR, NTYPE_CONST, NTYPE_UFUNC, NTYPE_BFUNC = 0, 1, 2, 3


class F:
    ADD = 1; SUB = 2; MUL = 3; DIV = 4; LOOSE_DIV = 5; POW = 6; LOOSE_POW = 7
    MAX = 8; MIN = 9; LT = 10; GT = 11; LE = 12; GE = 13
    SIN = 14; COS = 15; TAN = 16; SINH = 17; COSH = 18; TANH = 19
    LOG = 20; LOOSE_LOG = 21; EXP = 22; INV = 23; LOOSE_INV = 24
    NEG = 25; ABS = 26; SQRT = 27; LOOSE_SQRT = 28


def _sign0(a):
    return np.sign(a)   # sign(0) = 0, as the reference ABS rule (revad_interp.cuh:99)


def unary(f: int, a):
    """(value, d value / d a) of unary operator f (revad_interp.cuh:89-101)."""
    one = a.dtype.type(1)
    if f == F.SIN:
        return np.sin(a), np.cos(a)
    if f == F.COS:
        return np.cos(a), -np.sin(a)
    if f == F.TAN:
        r = np.tan(a); return r, one + r * r
    if f == F.SINH:
        return np.sinh(a), np.cosh(a)
    if f == F.COSH:
        return np.cosh(a), np.sinh(a)
    if f == F.TANH:
        r = np.tanh(a); return r, one - r * r
    if f == F.LOG:
        return np.log(a), one / a
    if f == F.LOOSE_LOG:
        return np.log(np.abs(a)), one / a
    if f == F.EXP:
        r = np.exp(a); return r, r
    if f in (F.INV, F.LOOSE_INV):
        r = one / a; return r, -r * r
    if f == F.NEG:
        return -a, np.full_like(a, -1)
    if f == F.ABS:
        return np.abs(a), _sign0(a)
    if f == F.SQRT:
        r = np.sqrt(a); return r, one / (a.dtype.type(2) * r)
    if f == F.LOOSE_SQRT:
        r = np.sqrt(np.abs(a)); return r, np.copysign(one / (a.dtype.type(2) * r), a)
    z = np.zeros_like(a)
    return z, z


def binary(f: int, l, r):
    """(value, d/d left, d/d right) of binary operator f (revad_interp.cuh:111-127)."""
    one = l.dtype.type(1)
    zero = np.zeros_like(l)
    if f == F.ADD:
        return l + r, np.ones_like(l), np.ones_like(l)
    if f == F.SUB:
        return l - r, np.ones_like(l), -np.ones_like(l)
    if f == F.MUL:
        return l * r, r, l
    if f in (F.DIV, F.LOOSE_DIV):
        o = l / r; return o, one / r, -o / r
    if f == F.POW:
        o = np.power(l, r)
        return o, r * np.power(l, r - one), o * np.log(l)
    if f == F.LOOSE_POW:
        al = np.abs(l); o = al ** r
        return o, r * np.power(al, r - one) * _sign0(l), o * np.log(al)
    if f == F.MAX:
        sel = (l >= r).astype(l.dtype)
        return np.maximum(l, r), sel, one - sel
    if f == F.MIN:
        sel = (l <= r).astype(l.dtype)
        return np.minimum(l, r), sel, one - sel
    if f == F.LT:
        return (l < r).astype(l.dtype), zero, zero
    if f == F.GT:
        return (l > r).astype(l.dtype), zero, zero
    if f == F.LE:
        return (l <= r).astype(l.dtype), zero, zero
    if f == F.GE:
        return (l >= r).astype(l.dtype), zero, zero
    return zero, zero, zero


def safe_mul(a, b):
    """Edge product with exact-zero annihilation (revad_interp.cuh:45-47)."""
    with np.errstate(all="ignore"):
        return np.where((a == 0) | (b == 0), a.dtype.type(0), a * b)


def eval_tree_arrays(nt, nv, ci, xs, c, dtype=np.float64):
    """Value of one tree at every row of xs (N, n_vars) with constants c (K,) -> (N,)."""
    y, _ = value_and_jacobian(nt, nv, ci, xs, c, dtype=dtype, jacobian=False)
    return y


def value_and_jacobian(nt, nv, ci, xs, c, dtype=np.float64, jacobian=True):
    """(y (N,), J (N, K)) with J[i, k] = d y_i / d c_k by the reverse sweep."""
    xs = np.asarray(xs, dtype)
    c = np.asarray(c, dtype).ravel()
    N = xs.shape[0]
    n = len(nt)
    K = c.size
    st: list = []
    d1: list = [None] * n
    d2: list = [None] * n
    with np.errstate(all="ignore"):
        for i in range(n - 1, -1, -1):
            t = int(nt[i])
            if t == NTYPE_VAR:
                st.append(xs[:, int(nv[i])])
            elif t == NTYPE_CONST:
                st.append(np.full(N, c[int(ci[i])], dtype))
            elif t == NTYPE_UFUNC:
                v, d = unary(int(nv[i]), st.pop())
                d1[i] = d
                st.append(v.astype(dtype, copy=False))
            elif t == NTYPE_BFUNC:
                l = st.pop()
                r = st.pop()
                o, dl, dr = binary(int(nv[i]), l, r)
                d1[i], d2[i] = dl, dr
                st.append(o.astype(dtype, copy=False))
            else:
                raise ValueError(f"unsupported node_type {t} at node {i}")
        if len(st) != 1:
            raise RuntimeError(f"malformed tree: stack depth {len(st)} != 1")
        y = st[0]
        if not jacobian:
            return y, None
        J = np.zeros((N, K), dtype)
        adj_st = [np.ones(N, dtype)]
        for i in range(n):
            t = int(nt[i])
            adj = adj_st.pop()
            if t == NTYPE_CONST:
                J[:, int(ci[i])] += adj
            elif t == NTYPE_UFUNC:
                adj_st.append(safe_mul(adj, np.asarray(d1[i], dtype)))
            elif t == NTYPE_BFUNC:
                adj_st.append(safe_mul(adj, np.asarray(d2[i], dtype)))   # right (deeper)
                adj_st.append(safe_mul(adj, np.asarray(d1[i], dtype)))   # left (top)
    return y, J


def tree_view(pop: dict, m: int):
    """(nt, nv, ci, y_row, K) of tree m; a 1-D ym is a row shared by every tree."""
    off, n, _c_off, K = (int(v) for v in pop["metas"][m])
    ym = np.asarray(pop["ym"])
    y = ym if ym.ndim == 1 else ym[m]
    return pop["nt"][off:off + n], pop["nv"][off:off + n], pop["ci"][off:off + n], y, K


def eval_pop_tree(pop: dict, m: int, c, dtype=np.float64):
    nt, nv, ci, _y, _K = tree_view(pop, m)
    return eval_tree_arrays(nt, nv, ci, pop["xs"], c, dtype)


def loss_pop(pop: dict, c_final) -> np.ndarray:
    """Per-tree fp64 0.5*sum r^2 at c_final; non-finite -> inf (cusr/benchmark/interp.py:89-102)."""
    M = int(pop["M"])
    out = np.full(M, np.inf)
    c_final = np.asarray(c_final, np.float64)
    for m in range(M):
        _off, _n, c_off, K = (int(v) for v in pop["metas"][m])
        try:
            y = eval_pop_tree(pop, m, c_final[c_off:c_off + K])
        except Exception:  # noqa: BLE001
            continue
        if np.all(np.isfinite(y)):
            r = y - np.asarray(tree_view(pop, m)[3], np.float64)
            out[m] = 0.5 * float(np.sum(r * r))
    return out


def intermediate_scale(nt, nv, ci, xs, c) -> np.ndarray:
    """Per-sample max |intermediate value| over the tree's nodes (fp64), the magnitude that
    bounds the rounding error of a finite-precision evaluation of the same expression."""
    xs = np.asarray(xs, np.float64)
    c = np.asarray(c, np.float64)
    N = xs.shape[0]
    st: list = []
    scale = np.zeros(N)
    with np.errstate(all="ignore"):
        for i in range(len(nt) - 1, -1, -1):
            t = int(nt[i])
            if t == NTYPE_VAR:
                v = xs[:, int(nv[i])]
            elif t == NTYPE_CONST:
                v = np.full(N, c[int(ci[i])])
            elif t == NTYPE_UFUNC:
                a = st.pop()
                v, _ = unary(int(nv[i]), a)
                scale = np.fmax(scale, np.abs(a))
            else:
                l = st.pop()
                r = st.pop()
                v, _, _ = binary(int(nv[i]), l, r)
                scale = np.fmax(scale, np.fmax(np.abs(l), np.abs(r)))
            scale = np.fmax(scale, np.abs(v))
            st.append(v)
    return scale


def error_scale(nt, nv, ci, xs, c) -> np.ndarray:
    """First-order rounding-error scale of evaluating the tree at each sample:
    S = sum over operator nodes n of |d f / d v_n| * |v_n| (fp64, absolute partials).
    A finite-precision evaluation with unit roundoff u differs from the exact value by about
    u * S (times a small constant for library transcendentals), however the value itself
    compares to S; S >> |f| flags an ill-conditioned sample (cancellation, cos(exp(big)))."""
    xs = np.asarray(xs, np.float64)
    c = np.asarray(c, np.float64)
    N = xs.shape[0]
    n = len(nt)
    vals: list = [None] * n
    d1: list = [None] * n
    d2: list = [None] * n
    st: list = []
    with np.errstate(all="ignore"):
        for i in range(n - 1, -1, -1):
            t = int(nt[i])
            if t == NTYPE_VAR:
                v = xs[:, int(nv[i])]
            elif t == NTYPE_CONST:
                v = np.full(N, c[int(ci[i])])
            elif t == NTYPE_UFUNC:
                v, d = unary(int(nv[i]), st.pop())
                d1[i] = np.abs(d)
            else:
                l = st.pop()
                r = st.pop()
                v, dl, dr = binary(int(nv[i]), l, r)
                d1[i], d2[i] = np.abs(dl), np.abs(dr)
            vals[i] = v
            st.append(v)
        S = np.zeros(N)
        adj_st = [np.ones(N)]
        for i in range(n):
            t = int(nt[i])
            adj = adj_st.pop()
            if t == NTYPE_UFUNC:
                S = S + np.nan_to_num(adj * np.abs(vals[i]), nan=np.inf)
                adj_st.append(adj * d1[i])
            elif t == NTYPE_BFUNC:
                S = S + np.nan_to_num(adj * np.abs(vals[i]), nan=np.inf)
                adj_st.append(adj * d2[i])
                adj_st.append(adj * d1[i])
    return S


def fd_jacobian(nt, nv, ci, xs, c, eps: float, dtype=np.float64) -> np.ndarray:
    """Forward-difference Jacobian (N, K) of the reference FD variant
    (cusr/kernel/batch_lm_ad.cu:95-132): h = eps*|c_k| (eps when c_k == 0), taken as the
    representable step (c_k + h) - c_k (eps again if that is 0), J[:, k] = (f(c + h e_k) -
    f(c)) / h, all in `dtype`."""
    c = np.asarray(c, dtype).ravel()
    T = np.dtype(dtype).type
    f0 = eval_tree_arrays(nt, nv, ci, xs, c, dtype=dtype)
    J = np.zeros((f0.shape[0], c.size), dtype)
    with np.errstate(all="ignore"):
        for k in range(c.size):
            saved = c[k]
            h = T(eps) * abs(saved)
            if h == 0:
                h = T(eps)
            cp = saved + h
            h = cp - saved
            if h == 0:
                h = T(eps)
            ck = c.copy()
            ck[k] = cp
            J[:, k] = (eval_tree_arrays(nt, nv, ci, xs, ck, dtype=dtype) - f0) / h
    return J


FAST_MATH_UNIT = 2.0 ** -21.41


def fast_math_error_scale(nt, nv, ci, xs, c) -> np.ndarray:
    """Error scale A of an fp32 evaluation built with nvcc --use_fast_math (the reference
    kernel's flags, cusr/kernel/Makefile:9): the result differs from the exact value by about
    FAST_MATH_UNIT * A beyond the rounding covered by error_scale. Per operator node, |d f /
    d v_n| times the published error of the intrinsic it maps to (CUDA C++ Programming Guide,
    intrinsic functions): __sinf / __cosf absolute 2^-21.41 on [-pi, pi], growing with |a|
    outside; __logf absolute 2^-21.41 on [0.5, 2], 3 ulp elsewhere; __expf (and the
    hyperbolics built on it) 2 + 1.173 |a| ulp; __powf through exp2(b log2 a); approximate
    division, reciprocal and square root 2 ulp."""
    xs = np.asarray(xs, np.float64)
    c = np.asarray(c, np.float64)
    N = xs.shape[0]
    n = len(nt)
    vals: list = [None] * n
    args: list = [None] * n
    d1: list = [None] * n
    d2: list = [None] * n
    st: list = []
    with np.errstate(all="ignore"):
        for i in range(n - 1, -1, -1):
            t = int(nt[i])
            if t == NTYPE_VAR:
                v = xs[:, int(nv[i])]
            elif t == NTYPE_CONST:
                v = np.full(N, c[int(ci[i])])
            elif t == NTYPE_UFUNC:
                a = st.pop()
                v, d = unary(int(nv[i]), a)
                args[i] = (a, None)
                d1[i] = np.abs(d)
            else:
                l = st.pop()
                r = st.pop()
                v, dl, dr = binary(int(nv[i]), l, r)
                args[i] = (l, r)
                d1[i], d2[i] = np.abs(dl), np.abs(dr)
            vals[i] = v
            st.append(v)
        A = np.zeros(N)
        adj_st = [np.ones(N)]
        for i in range(n):
            t = int(nt[i])
            if t not in (NTYPE_UFUNC, NTYPE_BFUNC):
                adj_st.pop()
                continue
            adj = adj_st.pop()
            f = int(nv[i])
            v = np.abs(vals[i])
            a = np.abs(args[i][0])
            if t == NTYPE_UFUNC:
                if f in (F.SIN, F.COS, F.TAN):
                    e = np.fmax(1.0, a) * (1.0 + (v * v if f == F.TAN else 0.0))
                elif f in (F.LOG, F.LOOSE_LOG):
                    e = 1.0 + v
                elif f in (F.EXP, F.SINH, F.COSH, F.TANH):
                    e = v * (1.0 + a)
                else:
                    e = v
                A = A + np.nan_to_num(adj * e, nan=np.inf)
                adj_st.append(adj * d1[i])
            else:
                if f in (F.POW, F.LOOSE_POW):
                    b = np.abs(args[i][1])
                    e = v * (1.0 + np.abs(np.log(np.fmax(a, 1e-300))) * b)
                else:
                    e = v
                A = A + np.nan_to_num(adj * e, nan=np.inf)
                adj_st.append(adj * d2[i])
                adj_st.append(adj * d1[i])
    return A


def intermediate_range(nt, nv, ci, xs, c):
    """Per-sample (max |v|, min nonzero |v|) over every node value of the tree (fp64): tells
    whether a narrower format can represent the evaluation at all (fp32 overflows above
    ~3.4e38 and loses precision below ~1.2e-38)."""
    xs = np.asarray(xs, np.float64)
    c = np.asarray(c, np.float64)
    N = xs.shape[0]
    st: list = []
    hi = np.zeros(N)
    lo = np.full(N, np.inf)
    with np.errstate(all="ignore"):
        for i in range(len(nt) - 1, -1, -1):
            t = int(nt[i])
            if t == NTYPE_VAR:
                v = xs[:, int(nv[i])]
            elif t == NTYPE_CONST:
                v = np.full(N, c[int(ci[i])])
            elif t == NTYPE_UFUNC:
                v, _ = unary(int(nv[i]), st.pop())
            else:
                l = st.pop()
                r = st.pop()
                v, _, _ = binary(int(nv[i]), l, r)
            a = np.abs(v)
            hi = np.fmax(hi, a)
            lo = np.where((a > 0) & np.isfinite(a), np.fmin(lo, a), lo)
            st.append(v)
    return hi, lo
