"""Restatement of the reference CPU backend ScipyPop. TEST / BASELINE INFRASTRUCTURE ONLY.

cusr/benchmark/backends.py:97-162: per tree, scipy.optimize.least_squares(method='lm',
xtol=1e-10, ftol=1e-10, max_nfev=200) on the fp64 residual f(x; c) - y with non-finite
residuals replaced by 1e6; a non-finite solution keeps c_init with status 2 (failed);
status 0 when scipy reports convergence (status >= 1), else 1; K = 0 trees are skipped
(status 3). Trees are fitted in a spawn pool (backends.py:31-68), one process per core.

The scipy algorithm itself (MINPACK lmdif: forward-difference Jacobian, trust-region LM) is
third-party code (scipy 1.18 here; the reference pins scipy 1.17.1 in uv.lock) and is used,
not restated.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time

import numpy as np

from . import interp

SETTINGS = dict(xtol=1e-10, ftol=1e-10, max_nfev=200)


def fit_one(payload):
    """(m, nt, nv, ci, xs, y, c0) -> (m, c_final fp64, status, nfev)."""
    from scipy.optimize import least_squares

    m, nt, nv, ci, xs, y, c0 = payload
    y64 = np.asarray(y, np.float64)

    def residual(c):
        r = interp.eval_tree_arrays(nt, nv, ci, xs, c) - y64
        return np.where(np.isfinite(r), r, 1e6)

    c0 = np.asarray(c0, np.float64)
    try:
        res = least_squares(residual, c0, method="lm", **SETTINGS)
        c = np.asarray(res.x, np.float64)
        if not np.all(np.isfinite(c)):
            return m, c0, 2, int(res.nfev)
        return m, c, (0 if res.status >= 1 else 1), int(res.nfev)
    except Exception:  # noqa: BLE001 — one bad tree must not abort the batch
        return m, c0, 2, 0


def _payloads(pop: dict, trees):
    for m in trees:
        nt, nv, ci, y, K = interp.tree_view(pop, int(m))
        if K == 0:
            continue
        c_off = int(pop["metas"][m][2])
        yield (int(m), nt, nv, ci, pop["xs"], y, pop["c_init"][c_off:c_off + K])


class Pool:
    """Persistent spawn pool of scipy workers (one process per core), so repeated timed fits
    do not pay process start-up (the reference keeps its pool alive the same way,
    backends.py:31-50)."""

    def __init__(self, nproc: int | None = None):
        self.nproc = int(nproc or os.cpu_count() or 1)
        self._pool = mp.get_context("spawn").Pool(processes=self.nproc) if self.nproc > 1 else None

    def warm(self) -> None:
        if self._pool is not None:
            self._pool.map(_noop, range(self.nproc), chunksize=1)

    def fit_pop(self, pop: dict, trees=None) -> dict:
        M = int(pop["M"])
        trees = np.arange(M) if trees is None else np.asarray(trees)
        c_final = np.asarray(pop["c_init"], np.float64).copy()
        status = np.full(M, 3, np.int32)
        nfev = np.zeros(M, np.int32)
        payloads = list(_payloads(pop, trees))
        for p in payloads:
            status[p[0]] = 2
        t0 = time.perf_counter()
        it = (self._pool.imap_unordered(fit_one, payloads, chunksize=1)
              if self._pool is not None and len(payloads) > 1 else map(fit_one, payloads))
        for m, c, s, nf in it:
            c_off, K = int(pop["metas"][m][2]), int(pop["metas"][m][3])
            c_final[c_off:c_off + K] = c
            status[m], nfev[m] = s, nf
        wall = time.perf_counter() - t0
        return dict(c_final=c_final, status=status, nfev=nfev, wall=wall, cores=self.nproc,
                    n_fitted=len(payloads))

    def close(self) -> None:
        if self._pool is not None:
            self._pool.terminate()
            self._pool = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


def _noop(x):
    return x


def fit_pop(pop: dict, nproc: int | None = None, trees=None) -> dict:
    """Fit the trees `trees` (default all) of a pop; returns fp64 c_final over the whole pop
    (unfitted trees keep c_init), status / nfev per tree, wall seconds and cores used."""
    with Pool(nproc) as pool:
        return pool.fit_pop(pop, trees)
