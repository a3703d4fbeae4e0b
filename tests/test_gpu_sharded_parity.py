"""Fit parity of the sample-sharded configuration (N = 10,000,000 samples) against the
reference's scipy fits (tests/golden/sharded_scipy.npz: the reference's ScipyPop on an 8-tree
sample, inputs regenerated from the seeded generator and checked against the stored digest).

The fits run on one GPU over all samples: sharding the samples over ranks changes only where
the per-tree sums are formed (test_gpu_sharded.py shows both ranks of a sharded fit equal to
a one-GPU fit up to the order of the sums), so this is the parity of the configuration.
Checked: the parity-grade mode (co_inproc.PARITY) reaches the reference fit on every tree;
the configuration's own mode (the reference LM, fp32, 30 iterations, one start) is reported
beside it with the reference fp64 losses at c_init, c_final and scipy's solution.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from _helpers import GOLDEN, write_report
from cusr_b200 import InProcessCO, co_inproc, multistart, synth
from oracle import interp

pytestmark = pytest.mark.gpu


def _digest(pop) -> str:
    h = hashlib.sha256()
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        h.update(np.ascontiguousarray(pop[k]).tobytes())
    return h.hexdigest()


def test_sharded_config_parity_vs_reference_scipy():
    z = np.load(GOLDEN / "sharded_scipy.npz")
    pop = synth.make_config("sharded", M=int(z["sharded/M"]), seed=11)
    assert int(pop["N"]) == 10_000_000
    assert _digest(pop) == str(z["sharded/digest"])
    ref = z["sharded/scipy/loss64"]
    K = np.asarray(pop["metas"])[:, 3]
    elig = (K > 0) & np.isfinite(ref)

    def within(c):
        ours = interp.loss_pop(pop, np.asarray(c, np.float64))
        return ours, ours <= ref * (1 + 1e-6) + 1e-12

    with InProcessCO(device_id=0) as co:
        single = co.optimize_ex(pop, max_iter=int(pop["max_iter"]), precision=pop["precision"])
        res = multistart.fit_multistart(co, pop, **multistart.preset_kwargs(co_inproc.PARITY))
    l_single, ok_single = within(single["c_final"])
    l_par, ok_par = within(res["c_final"])
    frac = float(np.mean(ok_par[elig]))
    bad = [int(m) for m in np.flatnonzero(elig & ~ok_par)]
    write_report("parity_sharded_fullN_vs_scipy.json", {
        "trees": int(pop["M"]), "N": int(pop["N"]), "n_eligible": int(elig.sum()),
        "parity_mode_within_1e-6_or_better": frac,
        "single_start_within_1e-6_or_better": float(np.mean(ok_single[elig])),
        "scipy_loss64": ref.tolist(), "parity_mode_loss64": l_par.tolist(),
        "single_start_loss64": l_single.tolist(),
        "init_loss64": np.asarray(z["sharded/init/loss64"]).tolist(),
        "divergent": bad, "ratios": {str(m): float(l_par[m] / ref[m]) for m in bad}})
    assert frac >= 1.0, bad
