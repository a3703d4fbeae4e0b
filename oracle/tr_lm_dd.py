"""Trust-region Levenberg-Marquardt (oracle/tr_lm.py's restatement of MINPACK lmder) with the
normal equations accumulated and factored in extended precision. TEST INFRASTRUCTURE ONLY.

The engine's double-double trust-region fits (CoOptions.tr_dd: dd_gram_kernel and
lm_tr_step_kernel_dd) form J^T J, J^T f and sum f^2 from the fp64 Jacobian with exact products
and double-double sums, and run the Cholesky factorisations and solves of the step in
double-double. This restatement does the same with mpmath at CUSR_ORACLE_DIGITS decimal digits
(default 32, about double-double's 106 bits): every J^T J entry is the correctly rounded sum
of exact products at that precision, and the linear algebra of lmpar runs at it too.

On trees whose Jacobian is rank-deficient to machine precision it reaches the fits scipy's
MINPACK (QR of J) reaches from the same start, where the fp64 normal equations of
oracle/tr_lm.py take the basic solution and stall (tests/test_oracle.py).
"""
from __future__ import annotations

import numpy as np

import os

import mpmath as mp

from . import interp

mp.mp.dps = int(os.environ.get("CUSR_ORACLE_DIGITS", "32"))
_msqrt = np.vectorize(mp.sqrt, otypes=[object])
_mpf = np.vectorize(mp.mpf, otypes=[object])


def NORM(v):
    """Euclidean norm at the working precision."""
    v = np.asarray(v, dtype=object).ravel()
    return mp.sqrt(mp.fsum(x * x for x in v))


def SQRT(x):
    return _msqrt(x) if isinstance(x, np.ndarray) else mp.sqrt(x)


SENTINEL = 1e6
DWARF = np.finfo(np.float64).tiny
EPS = np.finfo(np.float64).eps


def _chol(A):
    n = A.shape[0]
    L = np.array([[mp.mpf(0)] * A.shape[0] for _ in range(A.shape[0])], dtype=object)
    for j in range(n):
        s = A[j, j] - L[j, :j] @ L[j, :j]
        if not s > 0:
            return None
        L[j, j] = SQRT(s)
        for i in range(j + 1, n):
            L[i, j] = (A[i, j] - L[i, :j] @ L[j, :j]) / L[j, j]
    return L


def _pchol(A):
    """Symmetrically pivoted Cholesky: (L, perm, rank), stopping at a non-positive pivot."""
    n = A.shape[0]
    W = A.copy()
    perm = np.arange(n)
    L = np.array([[mp.mpf(0)] * A.shape[0] for _ in range(A.shape[0])], dtype=object)
    for j in range(n):
        d = np.array([W[i, i] - L[i, :j] @ L[i, :j] for i in range(j, n)])
        k = j + int(np.argmax(d))
        if not d[k - j] > 0:
            return L, perm, j
        if k != j:
            W[[j, k]] = W[[k, j]]
            W[:, [j, k]] = W[:, [k, j]]
            L[[j, k]] = L[[k, j]]
            perm[[j, k]] = perm[[k, j]]
        L[j, j] = SQRT(d[k - j])
        for i in range(j + 1, n):
            L[i, j] = (W[i, j] - L[i, :j] @ L[j, :j]) / L[j, j]
    return L, perm, n


def _fsub(L, b):
    y = np.array([mp.mpf(0)] * len(b), dtype=object)
    for i in range(len(b)):
        y[i] = (b[i] - L[i, :i] @ y[:i]) / L[i, i]
    return y


def _bsub(L, y):
    x = np.array([mp.mpf(0)] * len(y), dtype=object)
    for i in range(len(y) - 1, -1, -1):
        x[i] = (y[i] - L[i + 1:, i] @ x[i + 1:]) / L[i, i]
    return x


def lmpar(A, g, d, delta, par):
    """(par, p): the step p solving (A + par D^2) p = -g with |Dp| within Delta/10 of delta
    (or par = 0 when the Gauss-Newton step is inside), MINPACK lmpar's iteration."""
    n = len(g)
    L, perm, r = _pchol(A)
    x = np.array([mp.mpf(0)] * n, dtype=object)
    if r > 0:
        Lr = L[:r, :r]
        x[perm[:r]] = -_bsub(Lr, _fsub(Lr, g[perm][:r]))
    dxnorm = NORM(d * x)
    fp = dxnorm - delta
    if fp <= 0.1 * delta:
        return 0.0, x
    parl = 0.0
    if r == n:
        t = NORM(_fsub(L, (d * (d * x) / dxnorm)[perm]))
        parl = ((fp / delta) / t) / t
    gnorm = NORM(g / d)
    paru = gnorm / delta
    if paru == 0:
        paru = DWARF / min(delta, 0.1)
    par = min(max(par, parl), paru)
    if par == 0:
        par = gnorm / dxnorm
    it = 0
    while True:
        it += 1
        if par == 0:
            par = max(DWARF, 0.001 * paru)
        Lp = _chol(A + par * np.diag(d * d))
        guard = 0
        while Lp is None and guard < 64:   # indefinite by rounding: raise par
            par = max(2 * par, 1e-15 * np.max(np.abs(np.diag(A))) / np.min(d * d), DWARF)
            Lp = _chol(A + par * np.diag(d * d))
            guard += 1
        x = -_bsub(Lp, _fsub(Lp, g))
        dxnorm = NORM(d * x)
        temp, fp = fp, dxnorm - delta
        if abs(fp) <= 0.1 * delta or (parl == 0 and fp <= temp and temp < 0) or it == 10:
            return par, x
        t = NORM(_fsub(Lp, d * (d * x) / dxnorm))
        parc = ((fp / delta) / t) / t
        if fp > 0:
            parl = max(parl, par)
        if fp < 0:
            paru = min(paru, par)
        par = max(parl, par + parc)


def fit_tree(nt, nv, ci, xs, y, c0, max_nfev=200, ftol=1e-10, xtol=1e-10, gtol=1e-8,
             factor=100.0):
    """One tree: (c_final, info, nfev) with MINPACK's info codes (1/2/3 ftol/xtol, 4 gtol,
    5 maxfev, 6/7/8 tolerances at machine precision, -1 non-finite start, -2 non-finite
    Jacobian)."""
    y64 = np.asarray(y, np.float64)
    xs = np.asarray(xs)

    def fj(c, jac):
        # the reference scipy backend's residual (backends.py:105-110): a non-finite residual
        # is the sentinel 1e6, whose forward difference, and so Jacobian row, is 0
        v, J = interp.value_and_jacobian(nt, nv, ci, xs, np.asarray(c, np.float64), jacobian=jac)
        r = v - y64
        bad = ~np.isfinite(r)
        if bad.any():
            r = np.where(bad, SENTINEL, r)
            if J is not None:
                J = np.where(bad[:, None], 0.0, J)
        return r, J

    x = np.asarray(c0, np.float64).copy().astype(object)
    with np.errstate(all="ignore"):
        f, J = fj(x, True)
        nfev = 1
        fnorm = NORM(f)
        if not mp.isfinite(fnorm):
            return x, -1, nfev
        par, it, d = 0.0, 1, None
        while True:
            JM, fM = _mpf(J), _mpf(f)
            A, g = JM.T @ JM, JM.T @ fM
            if not (np.all(np.isfinite(A.astype(float))) and np.all(np.isfinite(g.astype(float)))):
                return x, -2, nfev
            acn = SQRT(np.array([max(v, mp.mpf(0)) for v in np.diag(A)], dtype=object))
            if it == 1:
                d = np.array([mp.mpf(1) if v == 0 else v for v in acn], dtype=object)
                xnorm = NORM(d * x)
                delta = factor * xnorm if xnorm != 0 else factor
            gnorm = 0.0
            if fnorm != 0:
                nz = acn != 0
                if nz.any():
                    gnorm = float(np.max(np.abs(g[nz] / fnorm) / acn[nz]))
            if gnorm <= gtol:
                return x, 4, nfev
            d = np.array([max(a, b) for a, b in zip(d, acn)], dtype=object)
            while True:
                par, p = lmpar(A, g, d, delta, par)
                xn = (x + p).astype(np.float64)
                pnorm = NORM(d * p)
                if it == 1:
                    delta = min(delta, pnorm)
                fn, _ = fj(xn, False)
                nfev += 1
                fnorm1 = NORM(fn)
                if not mp.isfinite(fnorm1):
                    fnorm1 = np.inf
                actred = 1 - (fnorm1 / fnorm) ** 2 if 0.1 * fnorm1 < fnorm else -1.0
                t1 = SQRT(max(p @ A @ p, 0.0)) / fnorm
                t2 = SQRT(par) * pnorm / fnorm
                prered = t1 * t1 + t2 * t2 / 0.5
                dirder = -(t1 * t1 + t2 * t2)
                ratio = actred / prered if prered != 0 else 0.0
                if ratio <= 0.25:
                    temp = 0.5 if actred >= 0 else 0.5 * dirder / (dirder + 0.5 * actred)
                    if 0.1 * fnorm1 >= fnorm or temp < 0.1:
                        temp = 0.1
                    delta = temp * min(delta, pnorm / 0.1)
                    par = par / temp
                elif par == 0 or ratio >= 0.75:
                    delta = pnorm / 0.5
                    par = 0.5 * par
                if ratio >= 1e-4:
                    x, f, fnorm = xn, fn, fnorm1
                    xnorm = NORM(d * x)
                    it += 1
                info = 0
                if abs(actred) <= ftol and prered <= ftol and 0.5 * ratio <= 1:
                    info = 1
                if delta <= xtol * xnorm:
                    info = 3 if info == 1 else 2
                if info:
                    return x, info, nfev
                if nfev >= max_nfev:
                    return x, 5, nfev
                if abs(actred) <= EPS and prered <= EPS and 0.5 * ratio <= 1:
                    return x, 6, nfev
                if delta <= EPS * xnorm:
                    return x, 7, nfev
                if gnorm <= EPS:
                    return x, 8, nfev
                if ratio >= 1e-4:
                    break
            _, J = fj(x, True)


def fit_pop(pop: dict, trees=None, **kw) -> dict:
    """Every tree (or `trees`): c_final (fp64, c_init for K = 0 and failed fits), info, nfev."""
    M = int(pop["M"])
    c_out = np.asarray(pop["c_init"], np.float64).copy()
    info = np.zeros(M, np.int32)
    nfev = np.zeros(M, np.int32)
    for m in (range(M) if trees is None else trees):
        nt, nv, ci, y, K = interp.tree_view(pop, int(m))
        if K == 0:
            continue
        off = int(pop["metas"][m][2])
        c, inf, nf = fit_tree(nt, nv, ci, pop["xs"], y, pop["c_init"][off:off + K], **kw)
        if np.all(np.isfinite(np.asarray(c, np.float64))):
            c_out[off:off + K] = c
        info[m], nfev[m] = inf, nf
    return {"c_final": c_out, "info": info, "nfev": nfev}
