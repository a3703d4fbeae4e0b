"""How reproducible is the reference fit itself? TEST INFRASTRUCTURE ONLY.

The parity criterion compares a fit's fp64 loss with ONE run of the reference CPU backend
(ScipyPop: scipy least_squares LM per tree, restated in oracle/scipy_lm.py). This module re-runs
that backend with its inputs moved by one float32 ulp — every c_init value, or every target
value — and reports the fraction of trees whose new fit is within 1e-6 relative of, or better
than, the original run: the level the reference reaches against itself when only rounding
changes. Trees with redundant constants (Jacobians rank-deficient to machine precision) take
rounding-driven steps in MINPACK, so on the mid / long / metric grammars a large share of
fits changes minimum under a one-ulp perturbation.

    python -m oracle.scipy_floor metric|pr1|mid|physics|long|scale
"""
from __future__ import annotations

import sys

import numpy as np

from . import interp, scipy_lm


def within(loss, ref, elig):
    return float(np.mean((loss <= ref * (1 + 1e-6) + 1e-12)[elig]))


def perturbation_floor(pop: dict, ref: np.ndarray, nproc: int | None = None) -> dict:
    """Fractions of trees within 1e-6 of (or better than) `ref` (the reference fit's fp64
    losses) for a plain re-run, c_init + 1 ulp and y + 1 ulp (float32 ulps)."""
    K = np.asarray(pop["metas"])[:, 3]
    elig = (K > 0) & np.isfinite(ref)
    out = {"trees": int(elig.sum())}
    runs = {"rerun": pop}
    p = dict(pop)
    p["c_init"] = np.nextafter(np.asarray(pop["c_init"], np.float32), np.float32(np.inf))
    runs["c_init+1ulp"] = p
    p = dict(pop)
    p["ym"] = np.nextafter(np.asarray(pop["ym"], np.float32), np.float32(np.inf))
    runs["y+1ulp"] = p
    with scipy_lm.Pool(nproc) as pool:
        pool.warm()
        for name, q in runs.items():
            res = pool.fit_pop(q)
            out[name] = within(interp.loss_pop(pop, res["c_final"]), ref, elig)
    return out


def _golden(name: str):
    from pathlib import Path

    g = Path(__file__).resolve().parents[1] / "tests" / "golden"
    sys.path.insert(0, str(g.parent))
    from _helpers import load_npz_pop

    if name == "metric":
        z = np.load(g / "metric_scipy.npz")
        return load_npz_pop(z, "pop"), z["scipy/loss64"]
    if name == "pr1":
        z = np.load(g / "pr1_scipy.npz")
        return load_npz_pop(z, "pop"), z["scipy/loss64"]
    z = np.load(g / "configs_scipy.npz")
    return load_npz_pop(z, name), z[f"{name}/scipy/loss64"]


if __name__ == "__main__":
    for name in sys.argv[1:] or ["pr1"]:
        pop, ref = _golden(name)
        print(name, perturbation_floor(pop, ref), flush=True)
