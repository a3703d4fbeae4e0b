"""Multi-start fits: every tree fitted from several starting points in one device batch, the
lowest final loss kept — the parity-grade mode.

The reference's LM schedule (co_lib.cu) and MINPACK's trust-region LM (the scipy backend the
parity criterion compares against, backends.py:100-120) often end in different local minima of
the same nonconvex problem, and even MINPACK itself, given the exact instead of the
finite-difference Jacobian, ends elsewhere on about one tree in six. Fitting every tree from a
few starts with both algorithms and keeping the best reaches the scipy fit or a better one on
almost every tree.

The start axis lives on the device (CoOptions.n_starts): the engine compiles and stores each
tree's program once, every fit of the tree shares it, the start points are generated on the
device from a counter-based generator, the best start is selected on the device, and trees
whose first-wave fits agree skip their later starts. `start_points` below is the host
restatement of that generator (the same formulas, for tests and for callers who want the
points themselves).
"""
from __future__ import annotations

import numpy as np

from .co_inproc import PARITY

KINDS = ("scale", "shift", "fresh1", "fresh3")   # start kinds after c_init, cycled


def _mix64(z: np.ndarray) -> np.ndarray:
    """SplitMix64 output function (Steele, Lea & Flood 2014), on uint64 arrays (wrapping)."""
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def start_normal(seed: int, m, s, k, j) -> np.ndarray:
    """Standard normal number j (0 or 1) of constant k of start s of tree m: two uniforms from
    SplitMix64 mixing of (seed, tree, start, constant) and the Box-Muller transform."""
    m = np.asarray(m, np.uint64)
    s = np.asarray(s, np.uint64)
    kj = np.asarray(2 * np.asarray(k, np.int64) + j, np.uint64)
    h = _mix64(np.uint64(seed) ^ _mix64(m))
    h = _mix64(h ^ ((s << np.uint64(32)) | kj))
    h2 = _mix64(h)
    u1 = ((h >> np.uint64(11)).astype(np.float64) + 0.5) * 2.0 ** -53
    u2 = (h2 >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2)


def start_points(pop: dict, starts: int, seed: int = 0) -> np.ndarray:
    """Start points of every (tree m, start s), flattened in fit order (m * starts + s, each
    with the tree's K constants): start 0 is c_init; start s >= 1 is, by (s - 1) mod 4, a
    log-normal scaling c * exp(z1 / 2) + z2 / 20, a shift c + (|c| + 1) z1 / 2, a fresh N(0, 1)
    or a fresh N(0, 9) draw. float32, as the engine stores them."""
    M, S = int(pop["M"]), int(starts)
    metas = np.asarray(pop["metas"], np.int64).reshape(M, 4)
    K = metas[:, 3]
    tree = np.repeat(np.arange(M), S * K)
    start = np.repeat(np.tile(np.arange(S), M), np.repeat(K, S))
    kk = (np.concatenate([np.tile(np.arange(k), S) for k in K]) if K.sum()
          else np.zeros(0, np.int64))
    c0 = np.asarray(pop["c_init"], np.float32).astype(np.float64)[metas[tree, 2] + kk]
    z1 = start_normal(seed, tree, start, kk, 0)
    z2 = start_normal(seed, tree, start, kk, 1)
    kind = np.where(start == 0, -1, (start - 1) % len(KINDS))
    v = c0.copy()
    v = np.where(kind == 0, c0 * np.exp(0.5 * z1) + 0.05 * z2, v)
    v = np.where(kind == 1, c0 + 0.5 * (np.abs(c0) + 1.0) * z1, v)
    v = np.where(kind == 2, z1, v)
    v = np.where(kind == 3, 3.0 * z1, v)
    return v.astype(np.float32)


# device memory one double-double call may take for its fits' per-sample Jacobians and values
DD_BATCH_BYTES = 16 << 30


def _dd_stage(co, pop: dict, ds: int, max_iter: int, xtol: float, seed: int, kw: dict) -> dict:
    """The double-double trust-region starts of every tree (CoOptions.tr_dd), in batches of
    consecutive trees so that a call keeps at most DD_BATCH_BYTES of per-sample Jacobians and
    values on the device; outputs in tree order."""
    from .popio import slice_pop

    M, N = int(pop["M"]), int(pop["N"])
    kmax = max(1, int(np.asarray(pop["metas"]).reshape(M, 4)[:, 3].max(initial=0)))
    per_tree = ds * (kmax + 1) * N * 8
    batch = max(1, int(DD_BATCH_BYTES // per_tree))
    call = dict(max_iter=max_iter, precision="fp64", xtol=xtol, algorithm="trust_region",
                n_starts=ds, tr_starts=ds, wave1=min(8, ds - 1) if ds > 1 else 0, seed=seed,
                tr_dd=True, **kw)
    if batch >= M:
        return co.optimize_ex(pop, **call)
    parts = [co.optimize_ex(slice_pop(pop, np.arange(a, min(a + batch, M))), **call)
             for a in range(0, M, batch)]
    return {k: np.concatenate([np.asarray(p[k]) for p in parts])
            for k in ("c_final", "status", "loss_final", "iters")}


def preset_kwargs(preset: dict = PARITY) -> dict:
    """fit_multistart keyword arguments of a preset dict (co_inproc.PARITY, PARITY_FAST,
    PARITY_FP64)."""
    return {("starts" if k == "n_starts" else k): v for k, v in preset.items() if k != "algorithm"}


def fit_multistart(co, pop: dict, starts: int = PARITY["n_starts"],
                   max_iter: int = PARITY["max_iter"], xtol: float = PARITY["xtol"],
                   precision: str = PARITY["precision"], seed: int = 0,
                   damping_floor: float = PARITY["damping_floor"],
                   tr_starts: int = PARITY["tr_starts"], wave1: int = PARITY["wave1"],
                   polish: bool = PARITY["polish"],
                   explore_precision: str | None = PARITY["explore_precision"],
                   explore_max_iter: int | None = PARITY["explore_max_iter"],
                   explore_tol: float | None = PARITY["explore_tol"],
                   polish_starts: int = PARITY["polish_starts"],
                   polish_max_iter: int | None = PARITY["polish_max_iter"],
                   dd_starts: int = PARITY["dd_starts"], **kw) -> dict:
    """Fit every tree of `pop` from `starts` starting points (the first is its c_init) in one
    device call (InProcessCO.optimize_ex with n_starts) and return the best start's
    c_final / status / loss_init / loss_final / iters with its index ('start').
    polish: a second device call continues every tree's best fit with the trust-region LM
    (from its constants rounded to the fp32 of the ABI) and keeps whichever is lower.

    explore_precision / explore_max_iter / explore_tol: run the multi-start call in another
    precision (e.g. "fp32": about five times faster), with its own evaluation budget and
    ftol = xtol; the polish then runs in `precision` with max_iter / xtol and its result is
    kept wherever it is finite and no worse.
    polish_starts: the polish call's starts per tree — the best fit itself and perturbations
    of it (the start kinds of the start axis, around the best), in one wave;
    polish_max_iter: its evaluation budget (default max_iter).
    dd_starts > 0 (precision fp64): a third call fits every tree again from its c_init and
    dd_starts - 1 generated starts with the trust-region LM on double-double normal equations
    (CoOptions.tr_dd), which keeps the small singular directions of rank-deficient Jacobians
    as MINPACK's QR does; the lowest final loss of the three calls is kept.

    Defaults: the parity preset (co_inproc.PARITY)."""
    algorithm = "trust_region" if tr_starts > 0 else kw.pop("algorithm", "reference")
    explore = explore_precision is not None and explore_precision != precision
    x_kw = dict(kw)
    if explore and explore_tol is not None:
        x_kw["ftol"] = explore_tol
    res = co.optimize_ex(pop, max_iter=explore_max_iter if explore and explore_max_iter else max_iter,
                         precision=explore_precision if explore else precision,
                         xtol=explore_tol if explore and explore_tol is not None else xtol,
                         damping_floor=damping_floor, algorithm=algorithm, n_starts=starts,
                         tr_starts=tr_starts, wave1=wave1, seed=seed, **x_kw)
    if not polish:
        return res
    stats = co.stats()
    again = dict(pop)
    with np.errstate(over="ignore"):            # fits that ran off to huge constants
        again["c_init"] = np.asarray(res["c_final"], np.float32)
    ps = max(1, int(polish_starts))
    pol = co.optimize_ex(again, max_iter=polish_max_iter or max_iter, precision=precision,
                         xtol=xtol, algorithm="trust_region", n_starts=ps, tr_starts=ps, wave1=0,
                         seed=seed + 1,
                         **{k: v for k, v in kw.items() if k in ("y_shared", "ftol", "gtol")})
    lp, lr = np.asarray(pol["loss_final"]), np.asarray(res["loss_final"])
    if explore:
        # the polish starts at the explore stage's (float32) constants and only accepts
        # improvements: its loss is the better one unless it failed; the two stages' losses
        # come from different precisions, hence the tolerance
        better = np.isfinite(lp) & (lp <= lr * (1 + 1e-5) + 1e-30)
    else:
        better = lp < lr
    M = int(pop["M"])
    K = np.asarray(pop["metas"], np.int64).reshape(M, 4)[:, 3]
    out = {k: np.where(better, pol[k], res[k]) for k in ("status", "loss_final", "iters")}
    out["loss_init"] = res["loss_init"]
    out["start"] = res.get("start", np.zeros(M, np.int32))
    out["polished"] = better
    out["c_final"] = np.where(np.repeat(better, K), pol["c_final"], res["c_final"])
    out["stats"] = stats
    if dd_starts > 0 and precision == "fp64":
        dd = _dd_stage(co, pop, int(dd_starts), max_iter, xtol, seed + 2,
                       {k: v for k, v in kw.items() if k in ("y_shared", "ftol", "gtol")})
        take = np.isfinite(dd["loss_final"]) & (np.asarray(dd["loss_final"]) < out["loss_final"])
        for k in ("status", "loss_final", "iters"):
            out[k] = np.where(take, dd[k], out[k])
        out["c_final"] = np.where(np.repeat(take, K), dd["c_final"], out["c_final"])
        out["dd"] = take
    return out
