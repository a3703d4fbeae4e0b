"""Benchmark-runner backend: the engine behind the reference's `fit_pop(pop) -> FitResult`
contract (cusr/benchmark/backends.py:81-89, 749-785), so `runner.make_backend` can hold it
where it holds `CudaKernelPop`.

Status codes follow the runner's convention (backends.py:5-8): 0 converged, 1 iteration
limit, 2 failed (FAIL_NAN and FAIL_CHOLESKY), 3 K=0 skipped — the same map the reference
applies to its kernel (backends.py:746).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

from .co_inproc import get_inproc_co

_STATUS_MAP = np.array([0, 1, 2, 3, 2], np.int32)   # engine STATUS_* -> runner status


@dataclass
class FitResult:
    backend: str
    c_final: np.ndarray          # (total_c,) float64
    status: np.ndarray           # (M,) int
    n_iter: np.ndarray           # (M,) int
    wall_e2e: float              # fit_pop entry -> constants back in host memory
    wall_core: float             # device time of the fit (CUDA events)
    meta: dict = field(default_factory=dict)


class B200Pop:
    """In-process engine backend. precision 'fp32' (the SFU arithmetic), 'fp32_fast' (the
    reference kernel's fast-math arithmetic) or 'fp64'; shared target rows are detected and
    uploaded once. starts > 1: the parity-grade multi-start fit (cusr_b200.multistart: the
    device start axis, trust-region starts; max_iter then defaults to 200)."""

    def __init__(self, max_iter: int | None = None, precision: str = "fp32", device_id: int = 0,
                 name: str | None = None, starts: int = 1):
        self.starts = max(1, int(starts))
        self.max_iter = int(max_iter if max_iter is not None else (200 if self.starts > 1 else 50))
        self.precision = precision
        self.device_id = int(device_id)
        self.name = name or (f"b200:{precision}" if self.starts == 1
                             else f"b200:{precision}:ms{self.starts}")

    def fit_pop(self, pop: dict) -> FitResult:
        t0 = time.perf_counter()
        co = get_inproc_co(self.device_id, "ad")
        ym = np.asarray(pop["ym"])
        shared = ym.ndim == 1 or (ym.shape[0] > 0 and bool(np.all(ym == ym[0])))
        if shared and ym.ndim == 2:
            pop = dict(pop)
            pop["ym"] = ym[0] if ym.shape[0] else ym.reshape(-1)
        if self.starts > 1:
            from . import multistart

            res = multistart.fit_multistart(co, pop, starts=self.starts, max_iter=self.max_iter,
                                            precision=self.precision,
                                            wave1=min(8, self.starts - 1))
        else:
            res = co.optimize_ex(pop, max_iter=self.max_iter, precision=self.precision,
                                 y_shared=shared)
        st = co.stats()
        raw = res["status"]
        return FitResult(self.name, res["c_final"].astype(np.float64), _STATUS_MAP[raw],
                         res["iters"].astype(np.int32), time.perf_counter() - t0,
                         st["device_ms"] / 1e3,
                         meta=dict(dtype=self.precision, raw_status_counts={
                             int(k): int(v) for k, v in zip(*np.unique(raw, return_counts=True))},
                             criteria=(f"reference LM (lambda0 1e-3), max_iter={self.max_iter}"
                                       if self.starts == 1 else
                                       f"{self.starts} starts (trust region + reference LM), "
                                       f"max_iter={self.max_iter}, best final loss")))
