"""Multi-start fits: each tree is fitted from several starting points in one device batch and
the best final loss is kept.

The reference's LM iteration (lambda schedule of co_lib.cu) and MINPACK's trust-region LM
(the scipy backend the parity criterion compares against, backends.py:100-120) often end in
different local minima of the same nonconvex problem. Fitting every tree from S starts — the
given c_init first, then points around it and fresh draws — and keeping the lowest final loss
reaches the scipy fit or a better one on most trees at a cost the GPU absorbs (PR1, 256
trees x 256 starts: one batch of 65,536 fits). The starts are deterministic for a seed.
"""
from __future__ import annotations

import numpy as np

from . import popio

# start kinds after the first (which is c_init itself), cycled: log-normal scaling of c_init,
# additive noise scaled by |c_init| + 1, fresh N(0, 1), fresh N(0, 3^2)
KINDS = ("scale", "shift", "fresh1", "fresh3")


def start_points(pop: dict, starts: int, seed: int = 0) -> np.ndarray:
    """Constants of the replicated population (tree m, start s at position m * starts + s),
    flattened in the replicated c_init order."""
    M, S = int(pop["M"]), int(starts)
    metas = np.asarray(pop["metas"], np.int64).reshape(M, 4)
    K_r = np.repeat(metas[:, 3], S)
    c_idx = popio._ranges(np.repeat(metas[:, 2], S), K_r)
    c0 = np.asarray(pop["c_init"], np.float64)[c_idx]
    s_of = np.repeat(np.tile(np.arange(S), M), K_r)          # start index of every constant
    rng = np.random.default_rng(seed)
    z1 = rng.standard_normal(c0.size)
    z2 = rng.standard_normal(c0.size)
    kind = np.where(s_of == 0, -1, (s_of - 1) % len(KINDS))
    c = c0.copy()
    sel = kind == 0
    c[sel] = c0[sel] * np.exp(0.5 * z1[sel]) + 0.05 * z2[sel]
    sel = kind == 1
    c[sel] = c0[sel] + 0.5 * (np.abs(c0[sel]) + 1.0) * z1[sel]
    sel = kind == 2
    c[sel] = z1[sel]
    sel = kind == 3
    c[sel] = 3.0 * z1[sel]
    return c.astype(np.float32)


def select_best(pop: dict, starts: int, res: dict) -> dict:
    """Per tree of `pop`, the start with the lowest finite final loss (ties: the earlier
    start). `res` is the fit of the replicated population."""
    M, S = int(pop["M"]), int(starts)
    metas = np.asarray(pop["metas"], np.int64).reshape(M, 4)
    K = metas[:, 3]
    lf = np.asarray(res["loss_final"], np.float64).reshape(M, S)
    key = np.where(np.isfinite(lf), lf, np.inf)
    best = np.argmin(key, axis=1)                            # first minimum: earlier start
    j = np.arange(M) * S + best
    K_r = np.repeat(K, S)
    coff_r = np.cumsum(K_r) - K_r
    c_idx = popio._ranges(coff_r[j], K)
    out = {"c_final": np.asarray(res["c_final"], np.float64)[c_idx],
           "status": np.asarray(res["status"]).reshape(M, S)[np.arange(M), best],
           "loss_init": np.asarray(res["loss_init"], np.float64).reshape(M, S)[:, 0],
           "loss_final": lf[np.arange(M), best],
           "start": best.astype(np.int32)}
    if "iters" in res:
        out["iters"] = np.asarray(res["iters"]).reshape(M, S)[np.arange(M), best]
    return out


def fit_multistart(co, pop: dict, starts: int = 256, max_iter: int = 200, xtol: float = 1e-10,
                   precision: str = "fp64", seed: int = 0, max_batch: int = 1 << 20,
                   damping_floor: float = 1e-3) -> dict:
    """Fit every tree of `pop` from `starts` starting points (the first is its c_init) with
    `co.optimize_ex` and keep the best. Trees are processed in batches of at most
    `max_batch` replicated fits. Returns c_final / status / loss_init / loss_final / iters
    of the chosen start and its index ('start').

    Defaults: the robust settings measured against the reference's scipy fits — 256 starts,
    200 iterations, xtol 1e-10. With damping_floor > 0 the first half of the starts (c_init
    among them) use the reference damping with the floor only as a fallback for systems it
    cannot factor, the second half the floored damping on every solve (the reference damping
    makes a tree with a zero Jacobian column fail with FAIL_CHOLESKY; the floor keeps it
    solvable, at the price of slower convergence elsewhere)."""
    M, S = int(pop["M"]), max(1, int(starts))
    per = max(1, max_batch // S)
    parts = []
    for lo in range(0, M, per):
        idx = np.arange(lo, min(M, lo + per))
        sub = pop if (lo == 0 and idx.size == M) else popio.slice_pop(pop, idx)
        pts = start_points(sub, S, seed + lo)
        if damping_floor > 0 and S > 1:
            # first half: reference damping, floor as fallback; second half: floor always
            Sa = (S + 1) // 2
            first = _start_mask(sub, S, Sa)
            res_a = co.optimize_ex(popio.replicate(sub, Sa, c_init=pts[first]),
                                   max_iter=max_iter, precision=precision, xtol=xtol,
                                   damping_floor=damping_floor)
            res_b = co.optimize_ex(popio.replicate(sub, S - Sa, c_init=pts[~first]),
                                   max_iter=max_iter, precision=precision, xtol=xtol,
                                   damping_floor=damping_floor, damping_always=True)
            res = _interleave(sub, Sa, S - Sa, res_a, res_b)
        else:
            res = co.optimize_ex(popio.replicate(sub, S, c_init=pts), max_iter=max_iter,
                                 precision=precision, xtol=xtol)
        parts.append(select_best(sub, S, res))
    if len(parts) == 1:
        return parts[0]
    return {k: np.concatenate([p[k] for p in parts]) for k in parts[0]}


def _start_mask(pop: dict, S: int, Sa: int) -> np.ndarray:
    """Per constant of the S-fold replicated population: True for starts s < Sa."""
    M = int(pop["M"])
    K = np.asarray(pop["metas"], np.int64).reshape(M, 4)[:, 3]
    return np.repeat(np.tile(np.arange(S) < Sa, M), np.repeat(K, S))


def _interleave(pop: dict, Sa: int, Sb: int, res_a: dict, res_b: dict) -> dict:
    """Results of the (Sa + Sb)-fold replicated population from the fits of its first Sa
    and last Sb starts of every tree."""
    M = int(pop["M"])
    K = np.asarray(pop["metas"], np.int64).reshape(M, 4)[:, 3]
    ca = np.asarray(res_a["c_final"], np.float64)
    cb = np.asarray(res_b["c_final"], np.float64)
    la, lb = K * Sa, K * Sb                               # constants per tree in each fit
    oa, ob = np.cumsum(la) - la, np.cumsum(lb) - lb
    parts = []
    for m in range(M):
        parts.append(ca[oa[m]:oa[m] + la[m]])
        parts.append(cb[ob[m]:ob[m] + lb[m]])
    out = {"c_final": np.concatenate(parts) if parts else np.zeros(0)}
    for k in ("status", "loss_init", "loss_final", "iters"):
        if k in res_a:
            out[k] = np.concatenate([np.asarray(res_a[k]).reshape(M, Sa),
                                     np.asarray(res_b[k]).reshape(M, Sb)], axis=1).reshape(-1)
    return out
