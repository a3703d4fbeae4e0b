"""The CPU oracle, pinned against the reference's own outputs: interpreter values from the
reference numpy interpreter, the reference reverse-AD Jacobian samples, the reference's host-
compiled interpreters (oracle/_ref, when built), the reference fixtures' known answers, and the
reference ScipyPop fits."""
from __future__ import annotations

import numpy as np
import pytest

from _helpers import GOLDEN, fixture_pop, fixture_truth, load_npz_pop, pop1000
from cusr_b200 import popio, synth
from oracle import interp, lm, ref_host, scipy_lm


def test_interp_matches_reference_values():
    z = np.load(GOLDEN / "interp_vectors.npz")
    pop = load_npz_pop(z, "pr1")
    for m in range(pop["M"]):
        off, K = int(pop["metas"][m][2]), int(pop["metas"][m][3])
        y = interp.eval_pop_tree(pop, m, pop["c_init"][off:off + K])
        np.testing.assert_array_equal(y, z["pr1/values"][m])
    p1000, _ = pop1000()
    for m in range(64):
        off, K = int(p1000["metas"][m][2]), int(p1000["metas"][m][3])
        y = interp.eval_pop_tree(p1000, m, p1000["c_init"][off:off + K])
        np.testing.assert_array_equal(y, z["pop1000/values"][m])


def test_jacobian_matches_reference_revad_samples():
    z = np.load(GOLDEN / "jac_sample.npz")
    for i in range(int(z["n"])):
        nt, nv, ci, c = z[f"{i}/nt"], z[f"{i}/nv"], z[f"{i}/ci"], z[f"{i}/c"]
        x = z[f"{i}/x"]
        _, J = interp.value_and_jacobian(nt, nv, ci, x, c.astype(np.float64))
        rev = z[f"{i}/rev"]
        ok = np.isfinite(rev) & np.isfinite(J)
        scale = np.maximum(np.abs(rev), 1.0)
        # reference samples are fp32 evaluations of the same rules
        assert np.all(np.abs(J[ok] - rev[ok]) <= 2e-4 * scale[ok]), i
        # where fp32 gives a finite gradient the fp64 restatement does too
        assert not np.any(np.isfinite(rev) & ~np.isfinite(J))


@pytest.mark.skipif(not ref_host.available(), reason="oracle/_ref not built")
def test_interp_matches_reference_host_build():
    ref = ref_host.RefHost()
    pop, _ = pop1000()
    from cusr_b200 import synth
    pops = [popio.slice_pop(pop, 60), synth.make_config("pr1", M=60, N=16, seed=5)]
    for p in pops:
        for m in range(int(p["M"])):
            nt, nv, ci, _y, K = interp.tree_view(p, m)
            if any(int(v) in (21, 24, 28, 5, 7) for v in nv[nt >= 2]):
                continue   # LOOSE ops are not part of the reference CUDA interpreter
            off = int(p["metas"][m][2])
            c = np.asarray(p["c_init"][off:off + K], np.float32)
            y64, J64 = interp.value_and_jacobian(nt, nv, ci, p["xs"][:16], c.astype(np.float64))
            S = interp.error_scale(nt, nv, ci, p["xs"][:16], c)
            for i in range(16):
                v, g = ref.value_and_grad(nt, nv, ci, p["xs"][i], c)
                if not np.isfinite(y64[i]) or S[i] > 1e3 * max(abs(y64[i]), 1.0):
                    continue
                assert abs(v - y64[i]) <= 1e-5 * abs(y64[i]) + 64 * 2.0 ** -24 * S[i]
                ok = np.isfinite(J64[i]) & np.isfinite(g)
                sc = max(1.0, float(np.max(np.abs(J64[i][ok]), initial=0.0)))
                assert np.all(np.abs(g[ok] - J64[i][ok]) <= 1e-3 * sc)


def test_lm_oracle_known_answer_fixture():
    pop = fixture_pop("pop_fixture")
    truth = fixture_truth("pop_fixture_truth.json")
    for dtype in (np.float64, np.float32):
        res = lm.fit_pop(pop, max_iter=50, dtype=dtype)
        for i, fx in enumerate(truth["fixtures"]):
            c = res["c_final"][fx["c_offset"]:fx["c_offset"] + fx["K"]]
            rel = np.linalg.norm(c - fx["c_true"]) / np.linalg.norm(fx["c_true"])
            assert res["status"][i] == lm.CONVERGED and rel < 5e-3, (fx["name"], rel)


def test_lm_oracle_stress_statuses():
    pop = fixture_pop("pop_fixture_stress")
    truth = fixture_truth("pop_fixture_stress_truth.json")
    res = lm.fit_pop(pop, max_iter=50, dtype=np.float32)
    assert [int(s) for s in res["status"]] == [f["expect_status"] for f in truth["fixtures"]]


def test_lm_oracle_op_fixture():
    pop = fixture_pop("pop_fixture_op")
    truth = fixture_truth("pop_fixture_op_truth.json")
    res = lm.fit_pop(pop, max_iter=50, dtype=np.float64)
    for i, fx in enumerate(truth["fixtures"]):
        c = res["c_final"][fx["c_offset"]:fx["c_offset"] + fx["K"]]
        rel = np.linalg.norm(c - fx["c_true"]) / np.linalg.norm(fx["c_true"])
        assert res["status"][i] == lm.CONVERGED and rel < 5e-3, fx["name"]


def test_lm_oracle_scale_fixture_tier1():
    truth = fixture_truth("pop_fixture_scale_truth.json")
    for f in truth["files"]:
        pop = fixture_pop(f["bin"][:-4])
        res = lm.fit_pop(pop, max_iter=50, dtype=np.float64)
        for i, fx in enumerate(f["fixtures"]):
            if fx["tier"] != 1:
                continue
            c = res["c_final"][fx["c_offset"]:fx["c_offset"] + fx["K"]]
            ct = np.asarray(fx["c_true"])
            rel = float(np.max(np.abs(c - ct) / np.maximum(np.abs(ct), 1e-30)))
            assert res["status"][i] == lm.CONVERGED and rel < 5e-3, (f["bin"], fx["name"], rel)


def test_lm_oracle_never_worse_than_init_fp64():
    pop, _ = pop1000()
    sub = popio.slice_pop(pop, 80)
    res = lm.fit_pop(sub, max_iter=50, dtype=np.float32)
    lf = interp.loss_pop(sub, res["c_final"])
    li = interp.loss_pop(sub, sub["c_init"].astype(np.float64))
    fin = np.isfinite(li)
    assert np.all(lf[fin] <= li[fin] * (1 + 1e-12) + 1e-300)


def test_scipy_restatement_matches_reference_scipy_fits():
    pop, g = pop1000()
    idx = np.arange(0, 1000, 25)
    res = scipy_lm.fit_pop(pop, nproc=1, trees=idx)
    for m in idx:
        off, K = int(pop["metas"][m][2]), int(pop["metas"][m][3])
        np.testing.assert_allclose(res["c_final"][off:off + K], g["scipy/c_final"][off:off + K],
                                   rtol=1e-9, atol=1e-12)
        assert res["status"][m] == g["scipy/status"][m]


def test_reference_kernel_golden_is_consistent():
    # the A100 goldens of the reference AD kernel reproduce their fp64 loss in the oracle
    pop, g = pop1000()
    lf = interp.loss_pop(pop, g["refkernel/c_final"].astype(np.float64))
    np.testing.assert_allclose(lf, g["refkernel/loss64"], rtol=1e-12)
    assert np.bincount(g["refkernel/status"], minlength=5).sum() == 1000


def test_fp32_honesty_fixture_matches_manifest_counts():
    """The committed copy of the reference's fp32-honesty fixtures: 17 problems, 257 trees,
    the manifest's baseline offender counts (AD 208, FD 57 serious)."""
    z = np.load(GOLDEN / "fp32_honesty.npz")
    assert len(z["names"]) == 17
    n = sum(int(z[f"f{i}/M"]) for i in range(17))
    ad = sum(int(z[f"f{i}/ad_serious"].sum()) for i in range(17))
    fd = sum(int(z[f"f{i}/fd_serious"].sum()) for i in range(17))
    assert (n, ad, fd) == (257, 208, 57)


def test_trust_region_restatement_follows_scipy_minpack():
    """oracle/tr_lm.py against the reference backend's own optimizer, scipy least_squares(
    method='lm') (MINPACK lmder), handed the same exact Jacobian: on trees whose Jacobian at
    c_init is of full rank (smallest singular value > 1e-8 of the largest) both take the same
    evaluations and end at the same loss; rank-deficient trees part ways by design (MINPACK's
    QR keeps rounding-size pivots, the restatement the basic solution)."""
    from scipy.optimize import least_squares

    from oracle import tr_lm

    z = np.load(GOLDEN / "pr1_scipy.npz")
    pop = load_npz_pop(z, "pop")
    same = []
    for m in range(0, int(pop["M"]), 2):
        nt, nv, ci, y, K = interp.tree_view(pop, m)
        if K == 0:
            continue
        off = int(pop["metas"][m][2])
        c0 = np.asarray(pop["c_init"][off:off + K], np.float64)
        _v, J = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c0)
        if not np.all(np.isfinite(J)):
            continue
        sv = np.linalg.svd(J, compute_uv=False)
        if not sv[-1] > 1e-8 * sv[0]:
            continue
        y64 = np.asarray(y, np.float64)

        # the reference backend's residual (non-finite -> 1e6) and its exact Jacobian (0 rows
        # at the sentinels), the objective both optimizers see
        def fun(c):
            r = interp.eval_tree_arrays(nt, nv, ci, pop["xs"], c) - y64
            return np.where(np.isfinite(r), r, 1e6)

        def jac(c):
            v, Jc = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c)
            return np.where(np.isfinite(v - y64)[:, None], Jc, 0.0)

        with np.errstate(all="ignore"):
            r = least_squares(fun, c0, jac=jac, method="lm", xtol=1e-10, ftol=1e-10,
                              max_nfev=200)
            c, _info, nfev = tr_lm.fit_tree(nt, nv, ci, pop["xs"], y, c0)
            ls = np.sum((interp.eval_tree_arrays(nt, nv, ci, pop["xs"], r.x) - y64) ** 2)
            lo = np.sum((interp.eval_tree_arrays(nt, nv, ci, pop["xs"], c) - y64) ** 2)
        same.append(abs(lo - ls) <= 1e-6 * abs(ls) and r.nfev == nfev)
    assert len(same) >= 40
    assert np.mean(same) >= 0.8, np.mean(same)


def test_lm_trajectory_sensitivity_to_summation_order():
    """The floor of any engine-vs-oracle comparison of the reference LM: the oracle against
    itself with only the order of its sums over samples changed (sequential per-chunk sums,
    as a chunked device reduction takes them), in fp64. Accept/reject decisions at a converged
    point compare two losses equal to rounding, so a last-bit change sends some trajectories
    to another iterate; on PR1 about one tree in ten ends more than 1e-6 apart and a few
    percent end in another status. The engine's fp64 agreement with the oracle
    (test_gpu_fit.test_fp64_trajectories_match_oracle_lm) sits at this floor."""
    pop = synth.make_config("pr1", seed=0)
    trees = np.arange(0, int(pop["M"]), 2)
    a = lm.fit_pop(pop, max_iter=50, dtype=np.float64, trees=trees)
    b = lm.fit_pop(pop, max_iter=50, dtype=np.float64, trees=trees, sum_chunk=256)
    la, lb = a["loss_final"], b["loss_final"]
    fin = np.isfinite(la)
    same = np.mean((np.abs(la - lb) <= 1e-6 * np.abs(la) + 1e-12)[fin])
    status = np.mean(a["status"] == b["status"])
    # initial losses differ by rounding only
    np.testing.assert_allclose(a["loss_init"], b["loss_init"], rtol=1e-13)
    assert 0.8 <= same < 0.99, same
    assert 0.9 <= status < 1.0, status


def test_reference_fit_reproducibility_floor():
    """The reference fit is not reproducible at the rounding level: ScipyPop re-run on PR1
    with every c_init moved by one float32 ulp ends within 1e-6 of (or better than) its own
    golden fit on only ~84% of trees, with the targets moved by one ulp on ~91% (a plain re-run:
    100%). On the mid / long / metric grammars the figures are lower still
    (`python -m oracle.scipy_floor NAME`). A fit that reaches >= 99% against one reference run
    is therefore better than the reference against itself."""
    from oracle import scipy_floor

    z = np.load(GOLDEN / "pr1_scipy.npz")
    out = scipy_floor.perturbation_floor(load_npz_pop(z, "pop"), z["scipy/loss64"])
    assert out["rerun"] == 1.0
    assert out["c_init+1ulp"] < 0.95 and out["y+1ulp"] < 0.97, out


def test_trust_region_double_double_restatement_reaches_minpack():
    """Metric-sample tree 53 has a Jacobian rank-deficient to machine precision at its start
    (the column-scaled J's two smallest singular values are ~1e-16). MINPACK (the reference
    scipy backend) fits it to a loss the fp64 normal-equation restatement misses by a factor
    of ~8 (its step takes the basic solution); the same algorithm with the normal equations at
    32 digits (oracle/tr_lm_dd.py, the arithmetic of the engine's tr_dd fits) reaches it."""
    from oracle import tr_lm, tr_lm_dd

    z = np.load(GOLDEN / "metric_scipy.npz")
    pop = load_npz_pop(z, "pop")
    ref = z["scipy/loss64"]
    m = 53
    nt, nv, ci, y, K = interp.tree_view(pop, m)
    off = int(pop["metas"][m][2])
    c0 = pop["c_init"][off:off + K]
    y64 = np.asarray(y, np.float64)

    def loss(c):
        f = interp.eval_tree_arrays(nt, nv, ci, pop["xs"], np.asarray(c, np.float64))
        return 0.5 * float(np.sum((f - y64) ** 2))

    with np.errstate(all="ignore"):
        l64 = loss(tr_lm.fit_tree(nt, nv, ci, pop["xs"], y, c0)[0])
        ldd = loss(tr_lm_dd.fit_tree(nt, nv, ci, pop["xs"], y, c0)[0])
    assert l64 > 2.0 * ref[m]
    assert ldd <= ref[m] * (1 + 1e-6)
