"""numpy restatement of the reference batched-LM iteration, one tree at a time.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows cusr/kernel/co_lib.cu (AD variant) step by step:
  * re-seed: c = c_init, lambda = 1e-3, K = 0 -> K0_SKIP (:284-305);
  * initial loss 0.5*sum r^2 at c_init; non-finite -> FAIL_NAN (:312-329);
  * per iteration (:343-483): J at c, JtJ / Jtr (lm_core.cuh:148-177); solve
    (JtJ with diag*(1+lambda)) delta = -Jtr by Cholesky (batch_lm_ad.cu:134-192; fp64 solve,
    the reference's SOLVE_FP64 form), s <= 0 -> lambda *= 10, > 1e12 -> FAIL_CHOLESKY;
    c_try = c + delta; non-finite loss_try -> FAIL_NAN; improvement first (loss_try <= loss
    -> accept, then |delta| < xtol(|c_try| + xtol) -> CONVERGED else lambda = max(0.1 lambda,
    1e-12)); reject -> lambda *= 10, > 1e12 -> FAIL_NAN (:438-455);
  * fp64 audit of fp32 fits (lm_core.cuh:299-351).
Jacobians come from the reverse sweep of oracle.interp (revad_interp.cuh rules).
"""
from __future__ import annotations

import numpy as np

from . import interp

CONVERGED, MAXITER, FAIL_NAN, K0_SKIP, FAIL_CHOLESKY = range(5)


def _cholesky_solve(A: np.ndarray, b: np.ndarray):
    """Row-oriented Cholesky + substitutions in the reference order; None if a pivot <= 0."""
    K = A.shape[0]
    L = A.copy()
    for j in range(K):
        s = L[j, j] - float(np.dot(L[j, :j], L[j, :j]))
        if s <= 0.0:
            return None
        L[j, j] = np.sqrt(s)
        for i in range(j + 1, K):
            L[i, j] = (L[i, j] - float(np.dot(L[i, :j], L[j, :j]))) / L[j, j]
    x = b.copy()
    for i in range(K):
        x[i] = (x[i] - float(np.dot(L[i, :i], x[:i]))) / L[i, i]
    for i in range(K - 1, -1, -1):
        x[i] = (x[i] - float(np.dot(L[i + 1:, i], x[i + 1:]))) / L[i, i]
    return x


def _chunked(fn, n, chunk):
    """fn(lo, hi) summed over sample ranges of `chunk` in sequence (chunk None: one range)."""
    if not chunk:
        return fn(0, n)
    acc = fn(0, min(chunk, n))
    for lo in range(chunk, n, chunk):
        acc = acc + fn(lo, min(lo + chunk, n))
    return acc


def fit_tree(nt, nv, ci, xs, y, c0, max_iter=50, dtype=np.float64, lambda0=1e-3, xtol=1e-6,
             sum_chunk=None):
    """LM fit of one tree. Returns (c_final, status, loss_init, loss_final, iters).
    sum_chunk: sums over samples (loss, JtJ, Jtr) taken as a sequence of per-chunk sums, the
    way a chunked device reduction orders them (None: numpy's order over all samples)."""
    T = np.dtype(dtype).type
    c = np.asarray(c0, dtype).copy()
    K = c.size
    y = np.asarray(y, dtype)
    with np.errstate(all="ignore"):
        f, J = interp.value_and_jacobian(nt, nv, ci, xs, c, dtype=dtype, jacobian=K > 0)
        r = f - y
        n = r.shape[0]
        loss = T(0.5) * T(_chunked(lambda a, b: np.sum(r[a:b] * r[a:b], dtype=dtype), n, sum_chunk))
    loss_init = loss
    if K == 0:
        return c, K0_SKIP, loss_init, loss, 0
    if not np.isfinite(loss):
        return c, FAIL_NAN, loss_init, loss, 0
    lam = T(lambda0)
    status = MAXITER
    iters = 0
    xt = T(xtol)
    for _ in range(max_iter):
        iters += 1
        with np.errstate(all="ignore"):
            JtJ = _chunked(lambda a, b: J[a:b].T @ J[a:b], n, sum_chunk).astype(np.float64)
            Jtr = _chunked(lambda a, b: J[a:b].T @ r[a:b], n, sum_chunk).astype(np.float64)
        A = JtJ.copy()
        A[np.diag_indices(K)] *= float(T(1) + lam)
        sol = _cholesky_solve(A, -Jtr) if np.all(np.isfinite(A)) else None
        if sol is None and np.all(np.isfinite(A)):
            lam = T(lam * T(10))
            if lam > T(1e12):
                status = FAIL_CHOLESKY
                break
            continue
        if sol is None:          # NaN normal equations: the step is NaN (s <= 0 is false)
            sol = np.full(K, np.nan)
        delta = sol.astype(dtype)
        c_try = (c + delta).astype(dtype)
        with np.errstate(all="ignore"):
            f_t, J_t = interp.value_and_jacobian(nt, nv, ci, xs, c_try, dtype=dtype)
            r_t = f_t - y
            loss_try = T(0.5) * T(_chunked(lambda a, b: np.sum(r_t[a:b] * r_t[a:b], dtype=dtype),
                                           n, sum_chunk))
        if not np.isfinite(loss_try):
            status = FAIL_NAN
            break
        dn = T(np.sqrt(np.sum(delta * delta, dtype=dtype)))
        cn = T(np.sqrt(np.sum(c_try * c_try, dtype=dtype)))
        if loss_try <= loss:
            c, loss, J, r = c_try, loss_try, J_t, r_t
            if dn < xt * (cn + xt):
                status = CONVERGED
                break
            lam = T(lam * T(0.1))
            if lam < T(1e-12):
                lam = T(1e-12)
        else:
            lam = T(lam * T(10))
            if lam > T(1e12):
                status = FAIL_NAN
                break
    return c, status, loss_init, loss, iters


def loss64(nt, nv, ci, xs, y, c) -> float:
    with np.errstate(all="ignore"):
        f = interp.eval_tree_arrays(nt, nv, ci, xs, np.asarray(c, np.float64))
        r = f - np.asarray(y, np.float64)
        return float(0.5 * np.sum(r * r))


def fit_pop(pop: dict, max_iter=50, dtype=np.float64, lambda0=1e-3, xtol=1e-6, audit=None,
            trees=None, sum_chunk=None) -> dict:
    """Fit every tree (or the subset `trees`) of a pop dict. fp32 fits get the fp64 audit
    unless audit=False. Returns arrays over the selected trees."""
    idx = np.arange(int(pop["M"])) if trees is None else np.asarray(trees)
    if audit is None:
        audit = np.dtype(dtype) == np.float32
    out_c, st, li, lf, its = [], [], [], [], []
    for m in idx:
        nt, nv, ci, y, K = interp.tree_view(pop, int(m))
        c_off = int(pop["metas"][m][2])
        c0 = np.asarray(pop["c_init"][c_off:c_off + K])
        c, s, l0, l1, it = fit_tree(nt, nv, ci, pop["xs"], y, c0, max_iter, dtype, lambda0, xtol,
                                    sum_chunk)
        if audit and K > 0:
            lf64 = loss64(nt, nv, ci, pop["xs"], y, c)
            li64 = loss64(nt, nv, ci, pop["xs"], y, c0)
            if not np.isfinite(lf64) or (np.isfinite(li64) and lf64 > li64):
                c = np.asarray(c0, dtype).copy()
                if s == CONVERGED:
                    s = MAXITER
                l1 = li64
        out_c.append(np.asarray(c, np.float64))
        st.append(s)
        li.append(float(l0))
        lf.append(float(l1))
        its.append(it)
    return dict(c_final=np.concatenate(out_c) if out_c else np.zeros(0), status=np.asarray(st),
                loss_init=np.asarray(li), loss_final=np.asarray(lf), iters=np.asarray(its))
