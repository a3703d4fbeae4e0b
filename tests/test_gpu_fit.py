"""Batched LM fits on the device through the C ABI: the reference's known-answer fixtures,
status semantics, parity with the oracle LM iteration and with the reference fits, the fp64
audit invariant, determinism, context reuse, and the error codes."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from _helpers import GOLDEN, fixture_pop, fixture_truth, load_npz_pop, pop1000, write_report
from cusr_b200 import InProcessCO, co_inproc, get_inproc_co, popio, synth
from oracle import interp, lm

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def co():
    c = InProcessCO(device_id=0)
    yield c
    c.teardown()


def _report(name, data):
    write_report(f"parity_{name}.json", data)


def _c(res, fx):
    return np.asarray(res["c_final"][fx["c_offset"]:fx["c_offset"] + fx["K"]], np.float64)


@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_known_answer_fixture(co, precision):
    pop = fixture_pop("pop_fixture")
    truth = fixture_truth("pop_fixture_truth.json")
    res = co.optimize_ex(pop, max_iter=50, precision=precision)
    for i, fx in enumerate(truth["fixtures"]):
        rel = np.linalg.norm(_c(res, fx) - fx["c_true"]) / np.linalg.norm(fx["c_true"])
        assert res["status"][i] == 0 and rel < 5e-3, (fx["name"], rel)


def test_reference_abi_known_answer_fixture(co):
    pop = fixture_pop("pop_fixture")
    truth = fixture_truth("pop_fixture_truth.json")
    res = co.optimize(pop, max_iter=50)
    assert res["c_final"].dtype == np.float32
    for i, fx in enumerate(truth["fixtures"]):
        rel = np.linalg.norm(_c(res, fx) - fx["c_true"]) / np.linalg.norm(fx["c_true"])
        assert res["status"][i] == 0 and rel < 5e-3


def test_op_fixture(co):
    pop = fixture_pop("pop_fixture_op")
    truth = fixture_truth("pop_fixture_op_truth.json")
    res = co.optimize_ex(pop, max_iter=50, precision="fp32")
    for i, fx in enumerate(truth["fixtures"]):
        rel = np.linalg.norm(_c(res, fx) - fx["c_true"]) / np.linalg.norm(fx["c_true"])
        assert res["status"][i] == 0 and rel < 5e-3, fx["name"]


@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_scale_fixture_tier1(co, precision):
    truth = fixture_truth("pop_fixture_scale_truth.json")
    for f in truth["files"]:
        pop = fixture_pop(f["bin"][:-4])
        res = co.optimize_ex(pop, max_iter=50, precision=precision)
        for i, fx in enumerate(f["fixtures"]):
            if fx["tier"] != 1:
                continue
            ct = np.asarray(fx["c_true"])
            rel = float(np.max(np.abs(_c(res, fx) - ct) / np.maximum(np.abs(ct), 1e-30)))
            assert res["status"][i] == 0 and rel < 5e-3, (f["bin"], fx["name"], rel)


@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_stress_statuses(co, precision):
    pop = fixture_pop("pop_fixture_stress")
    truth = fixture_truth("pop_fixture_stress_truth.json")
    res = co.optimize_ex(pop, max_iter=50, precision=precision)
    assert [int(s) for s in res["status"]] == [f["expect_status"] for f in truth["fixtures"]]
    # K = 0: nothing to fit, reported loss is the initial loss
    assert res["loss_final"][0] == res["loss_init"][0]


def test_fp64_trajectories_match_oracle_lm(co):
    """Same algorithm, same precision: final losses agree with the oracle's LM iteration."""
    pop = synth.make_config("pr1", seed=0)
    res = co.optimize_ex(pop, max_iter=50, precision="fp64")
    ref = lm.fit_pop(pop, max_iter=50, dtype=np.float64)
    lf, rf = res["loss_final"], ref["loss_final"]
    fin = np.isfinite(rf)
    same = np.abs(lf - rf) <= 1e-6 * np.abs(rf) + 1e-12
    better = lf <= rf * (1 + 1e-6) + 1e-12
    status_same = float(np.mean(res["status"] == ref["status"]))
    _report("pr1_fp64_vs_oracle_lm", {"same_1e-6": float(np.mean(same[fin])),
                                       "same_or_better": float(np.mean(better[fin])),
                                       "status_agreement": status_same})
    assert np.mean(better[fin]) >= 0.9
    assert status_same >= 0.85


def test_pr1_fit_parity_vs_reference_scipy(co):
    """North-star parity: final fp64 loss within 1e-6 relative of, or better than, the
    reference fp64 fit (numpy interpreter + scipy LM). Reported in full; asserted at the
    level the engine reaches (divergent fits are listed in the report)."""
    z = np.load(GOLDEN / "pr1_scipy.npz")
    pop = load_npz_pop(z, "pop")
    res = co.optimize_ex(pop, max_iter=50, precision="fp64")
    ours = interp.loss_pop(pop, res["c_final"])
    ref = z["scipy/loss64"]
    K = pop["metas"][:, 3]
    elig = (K > 0) & np.isfinite(ref)
    ok = ours <= ref * (1 + 1e-6) + 1e-12
    frac = float(np.mean(ok[elig]))
    tier_a = float(np.mean((ours <= np.maximum(1.005 * ref, ref + 1e-10))[elig]))
    bad = [int(m) for m in np.flatnonzero(elig & ~ok)]
    _report("pr1_fp64_vs_scipy", {"within_1e-6_or_better": frac, "tier_a_1.005": tier_a,
                                  "n_eligible": int(elig.sum()), "divergent": bad,
                                  "ratios": {str(m): float(ours[m] / ref[m]) for m in bad}})
    # measured: the reference LM iteration itself (oracle restatement, 50 iterations) reaches
    # ~0.67 here; divergent trees end in other local minima than MINPACK's
    assert frac >= 0.6


def _multistart_parity(co, name, pop, ref, **kw):
    """North-star parity with the parity-grade fit (cusr_b200.multistart defaults, the device
    start axis: 128 trust-region starts per tree explored in fp32 in two waves, then each
    tree's best polished in fp64 from 8 starts around it; the best final loss kept):
    the fraction of trees whose fp64 loss is within 1e-6 relative of, or better than, the
    reference scipy fit. Divergent trees are listed. The bars are the measured levels: on
    the mid grammar a few trees in a hundred keep a local minimum worse than MINPACK's, whose
    steps on Jacobians rank-deficient to machine precision are rounding-driven (the reference
    itself, re-run with its inputs moved by one ulp, reaches its own fit on 66-74% of mid
    trees: oracle/scipy_floor.py)."""
    from cusr_b200 import multistart

    res = multistart.fit_multistart(co, pop, **kw)
    st = res.get("stats") or co.stats()       # the multi-start call's (not the polish's)
    ours = interp.loss_pop(pop, res["c_final"])
    K = np.asarray(pop["metas"])[:, 3]
    elig = (K > 0) & np.isfinite(ref)
    ok = ours <= ref * (1 + 1e-6) + 1e-12
    frac = float(np.mean(ok[elig]))
    bad = [int(m) for m in np.flatnonzero(elig & ~ok)]
    _report(f"{name}_multistart_vs_scipy", {
        "within_1e-6_or_better": frac, "n_eligible": int(elig.sum()),
        "starts": int(st["n_starts"]), "fits_run": int(st["fits_run"]),
        "trees_retired": int(st["trees_retired"]), "device_ms": st["device_ms"],
        "strictly_better_than_scipy": float(np.mean((ours < ref * (1 - 1e-6))[elig])),
        "winning_start_histogram": np.bincount(res["start"], minlength=int(st["n_starts"])).tolist(),
        "divergent": bad, "ratios": {str(m): float(ours[m] / ref[m]) for m in bad}})
    return frac


def test_pr1_multistart_parity_vs_reference_scipy(co):
    """PR1 with its reference scipy fits (single start: 66%; measured 99.6%)."""
    z = np.load(GOLDEN / "pr1_scipy.npz")
    assert _multistart_parity(co, "pr1", load_npz_pop(z, "pop"), z["scipy/loss64"]) >= 0.99


def test_pop1000_multistart_parity_vs_reference_scipy(co):
    """The reference's own pop.bin fixture and its scipy fits."""
    pop, g = pop1000()
    assert _multistart_parity(co, "pop1000", pop, g["scipy/loss64"]) >= 0.99


@pytest.mark.parametrize("name,bar", [("mid", 0.98), ("physics", 0.99), ("long", 0.99),
                                      ("scale", 0.98)])
def test_config_multistart_parity_vs_reference_scipy(co, name, bar):
    """64-tree samples of the other BASELINE configurations (reduced N) with the reference's
    scipy fits (tests/golden/configs_scipy.npz); measured mid 96.9%, physics 100%, long 100%,
    scale 98.4-100% (one tree of 64 at 1.0036 in some start mixes)."""
    from cusr_b200 import multistart

    z = np.load(GOLDEN / "configs_scipy.npz")
    pop = load_npz_pop(z, name)
    kw = multistart.preset_kwargs(co_inproc.PARITY_MAX)
    assert _multistart_parity(co, name, pop, z[f"{name}/scipy/loss64"], **kw) >= bar


def _digest(pop):
    import hashlib

    h = hashlib.sha256()
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        h.update(np.ascontiguousarray(pop[k]).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name,bar", [("mid", 0.96), ("physics", 0.99), ("long", 0.93),
                                      ("scale", 0.96)])
def test_config_multistart_parity_full_n(co, name, bar):
    """32-tree samples of the configurations at their own N (mid 10,000, physics 100,000,
    long 4,096, scale 20,000) with the reference's scipy fits (configs_full_scipy.npz; the
    inputs are regenerated from the seeded generator and checked against the stored
    digest)."""
    z = np.load(GOLDEN / "configs_full_scipy.npz")
    pop = synth.make_config(name, M=int(z[f"{name}/M"]), seed=11)
    assert _digest(pop) == str(z[f"{name}/digest"])
    from cusr_b200 import multistart

    kw = multistart.preset_kwargs(co_inproc.PARITY_MAX)
    assert _multistart_parity(co, f"{name}_fullN", pop, z[f"{name}/scipy/loss64"], **kw) >= bar


def test_metric_sample_parity_modes(co):
    """The configuration behind the headline fits/s: a 256-tree stratified sample of the metric
    population at its full N = 10,000 with the reference's scipy fits (metric_scipy.npz).
    Reports the north-star fraction (fp64 loss within 1e-6 of, or better than, scipy) of the
    benchmarked single-start fp32 mode, of the reference's fast-math numerics, of fp64, of one
    trust-region start, and of the parity-grade multi-start fit."""
    from cusr_b200 import multistart

    z = np.load(GOLDEN / "metric_scipy.npz")
    pop = load_npz_pop(z, "pop")
    ref = z["scipy/loss64"]
    K = np.asarray(pop["metas"])[:, 3]
    elig = (K > 0) & np.isfinite(ref)

    def frac(c):
        blk = co.evaluate(pop, c=c, precision="fp64", values=False, blocks=True)["blocks"]
        l64 = np.array([b[-1] for b in blk])
        return float(np.mean((l64 <= ref * (1 + 1e-6) + 1e-12)[elig]))

    rep = {}
    for prec in ("fp32", "fp32_fast", "fp64"):
        rep[f"single_{prec}"] = frac(co.optimize_ex(pop, max_iter=50, precision=prec)["c_final"])
    rep["trust_region_fp64"] = frac(co.optimize_ex(pop, max_iter=200, precision="fp64",
                                                   xtol=1e-10, algorithm="trust_region")["c_final"])
    res = multistart.fit_multistart(co, pop)
    st = res.get("stats") or co.stats()
    rep["parity_mode"] = frac(res["c_final"])
    rep["parity_mode_fits_run"] = int(st["fits_run"])
    rep["parity_mode_trees_retired"] = int(st["trees_retired"])
    rep["parity_mode_device_ms"] = st["device_ms"]
    fast = multistart.fit_multistart(co, pop, **multistart.preset_kwargs(co_inproc.PARITY_FAST))
    rep["parity_fast"] = frac(fast["c_final"])
    rep["parity_fast_device_ms"] = fast["stats"]["device_ms"]
    f64 = multistart.fit_multistart(co, pop, **multistart.preset_kwargs(co_inproc.PARITY_FP64))
    rep["parity_fp64"] = frac(f64["c_final"])
    _report("metric_sample_modes_vs_scipy", rep)
    # measured: single fp32 52%, fp64 62%, one trust-region start 74%; the parity presets
    # (fp32 exploration + 8-start fp64 polish / single-start polish / all fp64) 99.2-99.6%
    assert rep["single_fp32"] >= 0.45 and rep["parity_mode"] >= 0.99, rep
    assert rep["parity_fast"] >= 0.98 and rep["parity_fp64"] >= 0.98, rep


def test_trust_region_fp64_matches_oracle(co):
    """One trust-region start per tree on PR1 (fp64, 200 evaluations, scipy's tolerances)
    against oracle/tr_lm.py, the CPU restatement of the same algorithm: the same final loss
    (within 1e-6) on most trees (the rest part at rounding level in chaotic trajectories), and
    the north-star fraction against scipy at the level the restatement reaches (0.82)."""
    from oracle import tr_lm

    z = np.load(GOLDEN / "pr1_scipy.npz")
    pop = load_npz_pop(z, "pop")
    res = co.optimize_ex(pop, max_iter=200, precision="fp64", xtol=1e-10,
                         algorithm="trust_region")
    orc = tr_lm.fit_pop(pop)
    ours = interp.loss_pop(pop, res["c_final"])
    theirs = interp.loss_pop(pop, orc["c_final"])
    ref = z["scipy/loss64"]
    K = pop["metas"][:, 3]
    fin = (K > 0) & np.isfinite(theirs) & np.isfinite(ref)
    same = np.abs(ours - theirs) <= 1e-6 * np.abs(theirs) + 1e-12
    better = ours <= theirs * (1 + 1e-6) + 1e-12
    vs_scipy = float(np.mean((ours <= ref * (1 + 1e-6) + 1e-12)[fin]))
    _report("pr1_trust_region_vs_oracle", {
        "same_1e-6": float(np.mean(same[fin])), "same_or_better": float(np.mean(better[fin])),
        "vs_scipy": vs_scipy,
        "oracle_vs_scipy": float(np.mean((theirs <= ref * (1 + 1e-6) + 1e-12)[fin])),
        "status": np.bincount(res["status"], minlength=5).tolist(),
        "iters_median": float(np.median(res["iters"]))})
    assert np.mean(same[fin]) >= 0.75
    assert vs_scipy >= 0.74


def test_start_axis_points_match_generator(co):
    """With max_iter = 0 every fit stops at its start point: each tree reports the start point
    of the start with the lowest initial loss, which must be the host restatement's point of
    that start (multistart.start_points), and start 0 is c_init."""
    from cusr_b200 import multistart

    pop = synth.make_config("pr1", M=64, N=300, seed=17)
    S, seed = 12, 99
    res = co.optimize_ex(pop, max_iter=0, precision="fp64", n_starts=S, seed=seed)
    pts = multistart.start_points(pop, S, seed)
    K = pop["metas"][:, 3]
    offs = np.concatenate([[0], np.cumsum(S * K)])
    for m in range(int(pop["M"])):
        s = int(res["start"][m])
        k = int(K[m])
        want = pts[offs[m] + s * k: offs[m] + (s + 1) * k]
        got = popio.tree_consts(pop, res["c_final"], m).astype(np.float32)
        # the device's double log / cos / exp may round differently from the host's by an
        # ulp before the cast to float
        assert np.all(np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32)) <= 1), m
    kk = K > 0
    assert np.all(res["loss_final"][kk] <= res["loss_init"][kk] * (1 + 1e-12) + 1e-300)


def test_waves_retire_agreeing_trees(co):
    """Two waves: trees whose first-wave fits agree skip the later starts; the outcome is as
    good as running every start on nearly all trees, for fewer fits."""
    from cusr_b200 import multistart

    z = np.load(GOLDEN / "pr1_scipy.npz")
    pop = load_npz_pop(z, "pop")
    all_at_once = multistart.fit_multistart(co, pop, wave1=0, polish=False)
    n_all = co.stats()["fits_run"]
    waved = multistart.fit_multistart(co, pop, polish=False)
    st = co.stats()
    assert st["trees_retired"] > 0 and st["fits_run"] < n_all
    la = interp.loss_pop(pop, all_at_once["c_final"])
    lw = interp.loss_pop(pop, waved["c_final"])
    fin = np.isfinite(la)
    assert np.mean((lw <= la * (1 + 1e-6) + 1e-12)[fin]) >= 0.97


def test_pop1000_vs_reference_kernel_golden(co):
    """The reference AD kernel's outputs on its own fixture (A100 goldens): our fp32 fit is
    as good or better in fp64 on most trees and never worse than c_init."""
    pop, g = pop1000()
    res = co.optimize(pop, max_iter=50)
    ours = interp.loss_pop(pop, res["c_final"].astype(np.float64))
    theirs = g["refkernel/loss64"]
    init = g["init/loss64"]
    K = pop["metas"][:, 3]
    elig = (K > 0) & np.isfinite(init)
    not_worse_than_init = ours[elig] <= init[elig] * (1 + 1e-9) + 1e-12
    as_good = ours <= theirs * (1 + 1e-3) + 1e-9
    sc = g["scipy/loss64"]
    vs_scipy = ours <= np.maximum(1.05 * sc, sc + 1e-10)
    _report("pop1000_vs_refkernel", {
        "as_good_as_refkernel": float(np.mean(as_good[elig])),
        "not_worse_than_init": float(np.mean(not_worse_than_init)),
        "within_1.05_scipy_ours": float(np.mean(vs_scipy[elig])),
        "within_1.05_scipy_refkernel": float(np.mean((theirs <= np.maximum(1.05 * sc, sc + 1e-10))[elig])),
        "status_ours": np.bincount(res["status"], minlength=5).tolist(),
        "status_refkernel": np.bincount(g["refkernel/status"], minlength=5).tolist()})
    assert np.all(not_worse_than_init)
    assert np.mean(as_good[elig]) >= 0.9


def test_pop1000_fast_math_vs_reference_kernel_golden(co):
    """CO_PREC_FP32_FAST reproduces the reference kernel's build numerics (--use_fast_math);
    on its own fixture the fits are as good as its A100 goldens on most trees, never worse
    than c_init (fp64 audit), and agree with its statuses about as often as the IEEE mode."""
    pop, g = pop1000()
    res = co.optimize_ex(pop, max_iter=50, precision="fp32_fast")
    acc = co.optimize_ex(pop, max_iter=50, precision="fp32")
    ours = interp.loss_pop(pop, res["c_final"])
    theirs = g["refkernel/loss64"]
    init = g["init/loss64"]
    K = pop["metas"][:, 3]
    elig = (K > 0) & np.isfinite(init)
    not_worse_than_init = ours[elig] <= init[elig] * (1 + 1e-9) + 1e-12
    as_good = ours <= theirs * (1 + 1e-3) + 1e-9
    same_status = np.mean(res["status"] == g["refkernel/status"])
    same_status_ieee = np.mean(acc["status"] == g["refkernel/status"])
    _report("pop1000_fast_vs_refkernel", {
        "as_good_as_refkernel": float(np.mean(as_good[elig])),
        "status_agreement_fast": float(same_status),
        "status_agreement_ieee": float(same_status_ieee),
        "status_fast": np.bincount(res["status"], minlength=5).tolist(),
        "status_refkernel": np.bincount(g["refkernel/status"], minlength=5).tolist()})
    assert np.all(not_worse_than_init)
    assert np.mean(as_good[elig]) >= 0.9


def test_fp32_audit_invariant(co):
    """Delivered constants are never worse than c_init in fp64 (lm_core.cuh:299-351)."""
    pop = synth.make_config("mid", M=512, N=2000, seed=5)
    res = co.optimize_ex(pop, max_iter=30, precision="fp32")
    lf = interp.loss_pop(pop, res["c_final"])
    li = interp.loss_pop(pop, pop["c_init"].astype(np.float64))
    fin = np.isfinite(li)
    assert np.all(lf[fin] <= li[fin] * (1 + 1e-9) + 1e-12)


def test_convergence_honesty(co):
    pop = synth.make_config("mid", M=512, N=2000, seed=6)
    res = co.optimize_ex(pop, max_iter=50, precision="fp32")
    conv = res["status"] == 0
    assert np.all(res["loss_final"][conv] <= res["loss_init"][conv] * (1 + 1e-4) + 1e-12)


def test_determinism(co):
    pop = synth.make_config("mid", M=300, N=3000, seed=8)
    a = co.optimize_ex(pop, max_iter=40, precision="fp32")
    b = co.optimize_ex(pop, max_iter=40, precision="fp32")
    for k in a:
        assert a[k].tobytes() == b[k].tobytes(), k


def test_reuse_across_sizes_matches_fresh_context(co):
    """Grow-only buffers across calls of changing M / K / N give the same results as a
    fresh context (the reference's in-process reuse suite, test_inproc_reuse.py)."""
    seq = [synth.make_config("mid", M=2000, N=500, seed=1),
           synth.make_config("pr1", M=40, N=1500, seed=2),
           synth.make_config("long", M=30, N=300, seed=3),
           synth.make_config("pr1", M=700, N=100, seed=4)]
    outs = [co.optimize_ex(p, max_iter=20, precision="fp32") for p in seq]
    fresh = InProcessCO(device_id=0)
    try:
        for p, o in zip(seq, outs):
            f = fresh.optimize_ex(p, max_iter=20, precision="fp32")
            for k in o:
                assert o[k].tobytes() == f[k].tobytes(), k
            fresh.teardown()
            fresh = InProcessCO(device_id=0)
    finally:
        fresh.teardown()


def test_loaded_fit_equals_one_shot(co):
    pop = synth.make_config("mid", M=400, N=1000, seed=9)
    a = co.optimize_ex(pop, max_iter=25, precision="fp32")
    co.load(pop, precision="fp32")
    b = co.fit_loaded(max_iter=25)
    c = co.fit_loaded(max_iter=25)
    for k in a:
        assert a[k].tobytes() == b[k].tobytes() == c[k].tobytes(), k


def test_reference_abi_matches_extended_entry(co):
    pop = synth.make_config("pr1", M=128, N=800, seed=10)
    a = co.optimize(popio.replicate_ym(pop), max_iter=30)
    b = co.optimize_ex(pop, max_iter=30, precision="fp32", y_shared=True)
    np.testing.assert_array_equal(a["c_final"], b["c_final"].astype(np.float32))
    np.testing.assert_array_equal(a["status"], b["status"])
    np.testing.assert_array_equal(a["loss_final"], b["loss_final"].astype(np.float32))


def test_singleton_and_reference_library_names():
    a = get_inproc_co(0, "ad")
    assert a is get_inproc_co(0, "ad")
    assert Path(co_inproc._so_path("ad")).resolve() == co_inproc.default_lib_path().resolve()
    out = a.optimize(fixture_pop("pop_fixture"), max_iter=50)
    assert set(out) == {"c_final", "status", "loss_init", "loss_final"}


def test_error_codes(co):
    pop = synth.make_config("pr1", M=10, N=50, seed=12)
    bad = dict(pop)
    bad["total_c"] = pop["total_c"] + 1
    with pytest.raises(co_inproc.COError) as e:
        co.optimize(bad)
    assert e.value.code == co_inproc.CO_ERR_SUM_C
    bad = dict(pop)
    bad["total_nodes"] = pop["total_nodes"] - 1
    with pytest.raises(co_inproc.COError) as e:
        co.optimize(bad)
    assert e.value.code == co_inproc.CO_ERR_SUM_NODES
    bad = dict(pop)
    bad["K_max"] = 33
    with pytest.raises(co_inproc.COError) as e:
        co.optimize(bad)
    assert e.value.code == co_inproc.CO_ERR_BOUNDS
    bad = dict(pop)
    bad["max_stack"] = 65
    with pytest.raises(co_inproc.COError) as e:
        co.optimize(bad)
    assert e.value.code == co_inproc.CO_ERR_BOUNDS
    bad = dict(pop)
    nt = pop["nt"].copy()
    nt[0] = 7
    bad["nt"] = nt
    with pytest.raises(co_inproc.COError) as e:
        co.optimize(bad)
    assert e.value.code == co_inproc.CO_ERR_BADTREE
    # the context survives errors
    assert co.optimize(pop, max_iter=5)["status"].shape == (10,)


def test_empty_population(co):
    pop = popio.build_pop([], np.zeros((5, 2), np.float32), np.zeros((0, 5), np.float32))
    out = co.optimize(pop)
    assert out["c_final"].size == 0 and out["status"].size == 0


def test_per_tree_targets_physics_fp64(co):
    pop = synth.make_config("physics", M=64, N=5000, seed=2)
    res = co.optimize_ex(pop, max_iter=100, precision="fp64")
    ref = lm.fit_pop(pop, max_iter=100, dtype=np.float64)
    better = res["loss_final"] <= ref["loss_final"] * (1 + 1e-6) + 1e-12
    assert np.mean(better) >= 0.9


def test_ad_modes_give_the_same_fits(co):
    """CoOptions.ad_mode: forward tangents (K <= 2) and the reverse sweep are two derivations
    of the same Jacobian; fp64 fits agree to rounding-driven trajectory differences."""
    pop = synth.make_config("pr1", M=256, N=1000, seed=9)
    rev = co.optimize_ex(pop, max_iter=50, precision="fp64", ad_mode="reverse")
    fwd = co.optimize_ex(pop, max_iter=50, precision="fp64", ad_mode="forward")
    Ks = np.asarray(pop["metas"])[:, 3]
    big = Ks > 2
    # trees with K > 2 take the reverse path in both runs: identical
    for key in ("status", "loss_final", "iters"):
        assert np.array_equal(np.asarray(rev[key])[big], np.asarray(fwd[key])[big]), key
    small = ~big
    assert np.mean(rev["status"][small] == fwd["status"][small]) >= 0.95
    a, b = rev["loss_final"][small], fwd["loss_final"][small]
    both = np.isfinite(a) & np.isfinite(b)
    rel = np.abs(a[both] - b[both]) / np.maximum(np.abs(a[both]), 1e-30)
    assert np.mean(rel <= 1e-6) >= 0.95


def test_fitresult_backend_single_and_multistart():
    """backends.B200Pop.fit_pop -> FitResult with the runner's fields and status convention
    (backends.py:81-89, 746); the multi-start backend is as good or better per tree."""
    from cusr_b200.backends import B200Pop

    pop = synth.make_config("pr1", M=64, N=400, seed=12)
    one = B200Pop(precision="fp64").fit_pop(pop)
    ms = B200Pop(precision="fp64", starts=20).fit_pop(pop)
    for r in (one, ms):
        assert r.c_final.shape == (pop["total_c"],) and r.status.shape == (64,)
        assert set(np.unique(r.status)) <= {0, 1, 2, 3}
        assert r.wall_core > 0 and r.wall_e2e >= r.wall_core
    l1 = interp.loss_pop(pop, one.c_final)
    l2 = interp.loss_pop(pop, ms.c_final)
    fin = np.isfinite(l1)
    assert np.mean(l2[fin] <= l1[fin] * (1 + 1e-9) + 1e-15) >= 0.95


def _honesty_pops():
    z = np.load(GOLDEN / "fp32_honesty.npz")
    for i, name in enumerate(z["names"]):
        yield str(name), load_npz_pop(z, f"f{i}"), z[f"f{i}/ad_serious"]


@pytest.mark.parametrize("precision,max_iter", [("fp32", 50), ("fp32_fast", 50),
                                                ("fp32_fast", 1000)])
def test_fp32_honesty_regression(co, precision, max_iter):
    """The reference's fp32-honesty regression (cusr/kernel/tests/fp32_honesty_regression):
    257 trees on which its fast-math AD kernel reports CONVERGED with c_final worse in exact
    fp64 than c_init (208 of them > 2x worse). The property: a tree reported converged must
    not be worse in fp64 than its start. Checked with the reference's own numerics
    (fp32_fast) as well as IEEE fp32; the fp64 audit keeps it."""
    conv_worse, serious_base, n = [], 0, 0
    for name, pop, ad_serious in _honesty_pops():
        res = co.optimize_ex(pop, max_iter=max_iter, precision=precision)
        l0 = interp.loss_pop(pop, pop["c_init"].astype(np.float64))
        lf = interp.loss_pop(pop, res["c_final"])
        for m in range(int(pop["M"])):
            n += 1
            serious_base += int(ad_serious[m])
            worse = (not np.isfinite(lf[m])) or lf[m] > l0[m] * (1 + 1e-6) + 1e-9
            if int(res["status"][m]) == 0 and worse:
                conv_worse.append((name, m, float(lf[m] / l0[m])))
    _report(f"fp32_honesty_{precision}_{max_iter}", {"trees": n, "reference_ad_serious": serious_base,
                                                     "converged_but_worse": conv_worse})
    assert n == 257 and serious_base == 208
    assert conv_worse == []


def test_many_chunk_fit_sums(co):
    """N of 300,000 (74 chunks per tree): the step's per-tree sums run as their own
    block-parallel kernel (chunk_sum_kernel). The fp64 loss elements it hands the step equal
    the oracle's losses at c_init and at c_final, and the fits follow the oracle's LM
    iteration (same algorithm, fp64) on the trees whose trajectory is not chaotic."""
    pop = synth.make_config("pr1", M=16, N=300_000, seed=4)
    res = co.optimize_ex(pop, max_iter=20, precision="fp64")
    li = interp.loss_pop(pop, np.asarray(pop["c_init"], np.float64))
    lf = interp.loss_pop(pop, res["c_final"])
    K = np.asarray(pop["metas"])[:, 3]
    fin = (K > 0) & np.isfinite(li)
    np.testing.assert_allclose(res["loss_init"][fin], li[fin], rtol=1e-11)
    ok = np.isfinite(lf) & fin
    np.testing.assert_allclose(res["loss_final"][ok], lf[ok], rtol=1e-10)
    ref = lm.fit_pop(pop, max_iter=20, dtype=np.float64, trees=np.arange(8))
    same = np.abs(res["loss_final"][:8] - ref["loss_final"]) <= 1e-6 * np.abs(ref["loss_final"]) + 1e-12
    assert np.mean(same[np.isfinite(ref["loss_final"])]) >= 0.6


def test_trust_region_double_double_on_rank_deficient_trees(co):
    """Trees whose Jacobian is rank-deficient to machine precision at their start (metric
    sample 53, long full-N 16): one trust-region start from c_init on double-double normal
    equations (CoOptions.tr_dd) reaches the reference scipy fit or better (measured 0.922 and
    0.749 of its loss, the levels of MINPACK with the exact Jacobian and of the 32-digit
    restatement oracle/tr_lm_dd.py, stable across summation orders), where the fp64 normal
    equations end 8 and 10,000 times above it. tr_dd is an fp64 option."""
    cases = []
    z = np.load(GOLDEN / "metric_scipy.npz")
    cases.append((load_npz_pop(z, "pop"), z["scipy/loss64"], [53]))
    zf = np.load(GOLDEN / "configs_full_scipy.npz")
    cases.append((synth.make_config("long", M=int(zf["long/M"]), seed=11), zf["long/scipy/loss64"], [16]))
    rep = {}
    for pop, ref, trees in cases:
        sub = popio.slice_pop(pop, np.asarray(trees))
        kw = dict(precision="fp64", max_iter=200, xtol=1e-10, ftol=1e-10, gtol=1e-8,
                  algorithm="trust_region")
        l64 = interp.loss_pop(sub, co.optimize_ex(sub, **kw)["c_final"])
        r1 = co.optimize_ex(sub, tr_dd=True, **kw)
        r2 = co.optimize_ex(sub, tr_dd=True, **kw)
        np.testing.assert_array_equal(r1["c_final"], r2["c_final"])      # fixed-order sums
        ldd = interp.loss_pop(sub, r1["c_final"])
        for i, t in enumerate(trees):
            rep[str(t)] = {"fp64": float(l64[i] / ref[t]), "dd": float(ldd[i] / ref[t])}
            assert ldd[i] <= ref[t] * (1 + 1e-6), rep
            assert l64[i] > 2.0 * ref[t], rep
    _report("trust_region_double_double", rep)
    with pytest.raises(co_inproc.COError):
        co.optimize_ex(popio.slice_pop(cases[0][0], 4), precision="fp32", algorithm="trust_region",
                       tr_dd=True)
