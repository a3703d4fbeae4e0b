"""The reference's own CUDA LM path (batch_lm_revad built from its sources for sm_100a) as a
comparison arm: the operator re-encoding it needs (CPU), and our fits against its fits on the
same trees (GPU, when the binary was built)."""
from __future__ import annotations

import numpy as np
import pytest

from _helpers import GOLDEN, load_npz_pop, write_report
from cusr_b200 import InProcessCO, synth
from oracle import interp, ref_gpu


def test_strict_ops_same_values():
    """log|x| / sqrt|x| re-encoded as LOG(ABS(x)) / SQRT(ABS(x)): same values at every sample,
    one extra node per loose operator, constants untouched."""
    pop = synth.make_config("pr1", M=48, N=300, seed=3)
    strict = ref_gpu.strict_ops(pop)
    n_loose = int(np.sum((pop["nt"] == 2) & np.isin(pop["nv"], (21, 28))))
    assert n_loose > 0
    assert strict["total_nodes"] == pop["total_nodes"] + n_loose
    assert not np.any((strict["nt"] == 2) & np.isin(strict["nv"], (21, 28)))
    np.testing.assert_array_equal(strict["metas"][:, 2:], pop["metas"][:, 2:])
    for m in range(int(pop["M"])):
        a = interp.tree_view(pop, m)
        b = interp.tree_view(strict, m)
        c = pop["c_init"][pop["metas"][m][2]:pop["metas"][m][2] + pop["metas"][m][3]]
        va = interp.eval_tree_arrays(a[0], a[1], a[2], pop["xs"], c.astype(np.float64))
        vb = interp.eval_tree_arrays(b[0], b[1], b[2], pop["xs"], c.astype(np.float64))
        np.testing.assert_array_equal(va, vb)


def test_limits_checked_before_running():
    pop = synth.make_config("long", M=4, N=64, seed=1)        # trees up to 255 nodes, K up to 32
    why = ref_gpu.within_limits(ref_gpu.strict_ops(pop))
    assert why is not None and "MAX_NODES" in why


@pytest.mark.gpu
def test_fits_vs_reference_cuda_kernel():
    """The 256-tree sample of the metric population (N = 10,000): the reference kernel and our
    engine (IEEE fp32 and the reference's fast-math numerics), 50 iterations each; the fp64
    loss at every delivered c_final, compared per tree and against the reference scipy fit."""
    if not ref_gpu.BINARY.exists():
        pytest.skip("reference binary not built (make -C oracle)")
    z = np.load(GOLDEN / "metric_scipy.npz")
    pop = load_npz_pop(z, "pop")
    sc = z["scipy/loss64"]
    with ref_gpu.RefGPU(pop) as rg:
        ref = rg.run(max_iter=50)
    with InProcessCO(device_id=0) as co:
        def loss64(c):
            blk = co.evaluate(pop, c=c, precision="fp64", values=False, blocks=True)["blocks"]
            return np.array([b[-1] for b in blk])

        l_ref = loss64(ref["c_final"].astype(np.float64))
        ours = {p: co.optimize_ex(pop, max_iter=50, precision=p) for p in ("fp32", "fp32_fast")}
        l_ours = {p: loss64(r["c_final"]) for p, r in ours.items()}
    K = pop["metas"][:, 3]
    fin = (K > 0) & np.isfinite(sc)

    def as_good(a, b):
        return float(np.mean((a <= b * (1 + 1e-6) + 1e-12)[fin]))

    rep = {"trees": int(fin.sum()),
           "reference_kernel_vs_scipy": as_good(l_ref, sc),
           "reference_status": np.bincount(ref["status"], minlength=5).tolist()}
    for p in ours:
        rep[f"{p}_vs_scipy"] = as_good(l_ours[p], sc)
        rep[f"{p}_as_good_as_reference_kernel"] = as_good(l_ours[p], l_ref)
        rep[f"{p}_status_agreement"] = float(np.mean(ours[p]["status"] == ref["status"]))
        rep[f"{p}_status"] = np.bincount(ours[p]["status"], minlength=5).tolist()
    write_report("parity_vs_reference_kernel_metric.json", rep)
    # Same algorithm, different rounding: fp32 trajectories of nonconvex fits part ways on a
    # quarter of the trees (measured: 73-78% of trees as good as the reference kernel's, per
    # tree), so the comparison is over the population: against the reference scipy fit, the
    # fraction of trees as good or better is the reference kernel's, up to sampling noise.
    for p in ours:
        assert rep[f"{p}_vs_scipy"] >= rep["reference_kernel_vs_scipy"] - 0.06, rep
        assert rep[f"{p}_as_good_as_reference_kernel"] >= 0.6, rep
