"""The FD variant's library (libcusr_co_fd.so, the name the reference loader opens for
variant "fd" — get_inproc_co's default): co_optimize with the reference FD variant's
acceptance order (cusr/kernel/co_lib.cu:456-471: a step below xtol is CONVERGED and kept
before the improvement test; an improvement must be strict), checked on the reference's
known-answer fixtures and against the reference FD variant's own outputs on its pop.bin
fixture (cusr/kernel/tests/golden/fd/pop1000, A100 fast-math: statuses compared as
statistics, not bytes)."""
from __future__ import annotations

import numpy as np
import pytest

from _helpers import GOLDEN, fixture_pop, fixture_truth, pop1000, write_report
from cusr_b200 import co_inproc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fd():
    c = co_inproc.InProcessCO(device_id=0, lib_path=str(co_inproc._so_path("fd")), variant="fd")
    yield c
    c.teardown()


def test_fd_known_answers(fd):
    pop = fixture_pop("pop_fixture")
    truth = fixture_truth("pop_fixture_truth.json")
    res = fd.optimize(pop, max_iter=50)
    assert set(res) == {"c_final", "status"}          # the fd variant returns no losses
    for i, fx in enumerate(truth["fixtures"]):
        c = res["c_final"][fx["c_offset"]:fx["c_offset"] + fx["K"]].astype(np.float64)
        rel = np.linalg.norm(c - fx["c_true"]) / np.linalg.norm(fx["c_true"])
        assert res["status"][i] == 0 and rel < 5e-3, (fx["name"], rel)
    stress = fixture_pop("pop_fixture_stress")
    st = fd.optimize(stress, max_iter=50)["status"]
    want = [f["expect_status"] for f in fixture_truth("pop_fixture_stress_truth.json")["fixtures"]]
    assert st.tolist() == want


def test_fd_statuses_match_reference_fd_variant(fd):
    pop, _g = pop1000()
    gold = np.load(GOLDEN / "fd_pop1000.npz")
    res = fd.optimize(pop, max_iter=50)
    ad = co_inproc.InProcessCO(device_id=0).optimize(pop, max_iter=50)
    ours, ref = np.bincount(res["status"], minlength=5), np.bincount(gold["status"], minlength=5)
    agree = float(np.mean(res["status"] == gold["status"]))
    write_report("fd_variant_pop1000.json", {"ours": ours.tolist(), "reference_fd": ref.tolist(),
                                             "ad_ordering": np.bincount(ad["status"], minlength=5).tolist(),
                                             "status_agreement": agree})
    # The FD order converges more trees than the AD order (the reference's own goldens: 424 vs
    # 329 of 1000; measured here 489 vs 326). The engine's Jacobian is exact where the
    # reference FD variant's is a forward difference, so fewer systems fail to factor (78 vs
    # 138 FAIL_CHOLESKY) and more trees converge; statuses agree on 80% of trees.
    assert ours[0] > np.bincount(ad["status"], minlength=5)[0]
    assert abs(int(ours[0]) - int(ref[0])) <= 0.25 * ref[0]
    assert ours[3] == ref[3]                                # K = 0 trees
    assert agree >= 0.75, agree
