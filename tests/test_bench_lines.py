"""The bench line's derived fields, on the CPU with made-up engine counters: the live
roofline of a configuration (which stream counts as HBM traffic, which roof binds), the
north-star fraction and the fixtures the fit-parity fields read."""
from __future__ import annotations

import numpy as np
import pytest

import bench
from cusr_b200 import synth

COUNTERS = {"eval_ms": 1000.0, "flops": 7.0e12, "node_evals": 1e12, "sample_evals": 1e10,
            "eval_launches": 250}
PEAKS = (70.0, 35.0)     # fp32, fp64 TFLOP/s


def test_shared_target_in_l2_is_fp_bound():
    pop = synth.make_config("mid", M=16, N=1000, seed=0)
    r = bench.config_roofline(COUNTERS, pop, "fp32", PEAKS)
    assert r["bound"] == "fp32" and "hbm" not in r and "hbm_note" in r
    assert r["achieved"] == pytest.approx(7.0) and r["frac"] == pytest.approx(0.1)
    assert r["avg_launch_ms"] == pytest.approx(4.0)


def test_per_tree_targets_count_four_bytes_per_tree_sample():
    pop = synth.make_config("physics", M=16, N=1000, seed=0)
    r = bench.config_roofline(COUNTERS, pop, "fp64", PEAKS)
    hpk, _ = bench.measured_hbm_peak()
    assert r["fp"]["peak"] == 35.0
    assert r["hbm"]["achieved"] == pytest.approx(4 * 1e10 / 1e9)
    assert r["hbm"]["frac"] == pytest.approx(40.0 / hpk)
    assert r["bound"] == "fp64"                # 0.2 of the fp64 roof against 40 GB/s


def test_inputs_beyond_l2_stream_the_input_row_and_target():
    # 7,000,000 samples x (4 inputs + target) x 4 B = 140 MB > the 126 MB L2
    pop = synth.make_config("sharded", M=2, N=7_000_000, seed=0)
    slow = dict(COUNTERS, flops=1e9)
    r = bench.config_roofline(slow, pop, "fp32", PEAKS)
    per = 4 * (int(pop["n_vars"]) + 1)
    assert r["hbm"]["achieved"] == pytest.approx(per * 1e10 / 1e9)
    assert r["bound"] == "hbm"


def test_no_evaluation_time_is_reported_not_divided():
    pop = synth.make_config("mid", M=4, N=100, seed=0)
    r = bench.config_roofline(dict(COUNTERS, eval_ms=0.0), pop, "fp32", PEAKS)
    assert "unavailable" in r


class _FakeCO:
    """evaluate() returning fixed fp64 losses as the last block entry of every tree."""

    def __init__(self, losses):
        self.losses = losses

    def evaluate(self, pop, c, precision, values, blocks):
        assert precision == "fp64" and blocks and not values
        return {"blocks": [np.array([0.0, l]) for l in self.losses]}


def test_north_star_fraction_counts_fitted_trees_with_a_finite_reference():
    metas = np.array([[0, 3, 0, 1], [3, 3, 1, 1], [6, 1, 2, 0], [7, 3, 2, 1]], np.int32)
    sample = {"metas": metas}
    ref = np.array([1.0, 2.0, 5.0, np.nan])
    # tree 0 equal within 1e-6, tree 1 worse, tree 2 has K = 0, tree 3 has no reference fit
    co = _FakeCO([1.0 + 5e-7, 2.1, 0.0, 0.0])
    assert bench.north_star_fraction(co, sample, ref, c_final=None) == pytest.approx(0.5)


def test_metric_scipy_sample_is_the_committed_fixture():
    sample, ref = bench.metric_scipy_sample()
    assert sample is not None
    assert int(sample["M"]) == len(ref) == np.asarray(sample["metas"]).shape[0]
    assert int(sample["N"]) == 10_000
