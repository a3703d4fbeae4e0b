"""Generate the golden fixtures under tests/golden/ from the reference checkout.

Run in a container where the reference (TensorConv/CuSR) is importable:

    CUSR_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Everything written here comes from the reference's own code and files:
  fixtures.npz / fixtures.json   the reference's known-answer populations
                                 (cusr/kernel/tests/pop_fixture*.bin) and their truth JSONs
  pop1000.npz                    data/fixtures/pop.bin (M=1000, N=1000, shared y stored once),
                                 the reference AD kernel's A100 outputs for it
                                 (cusr/kernel/tests/golden/ad/pop1000/*.bin), the reference
                                 fp64 loss of both (cusr/benchmark/interp.loss_pop), and the
                                 reference scipy fits (cusr.benchmark.backends.ScipyPop)
  interp_vectors.npz             reference interpreter values (interp.eval_tree_arrays, fp64)
                                 on PR1-config trees from cusr_b200.synth and on pop1000
  pr1_scipy.npz                  reference ScipyPop fits of the PR1 configuration (seed 0)
  configs_scipy.npz              reference ScipyPop fits of 64-tree samples of the mid,
                                 physics, long and scale configurations (seed 7, reduced N)
  fp32_honesty.npz               the reference's fp32-honesty regression fixtures
                                 (cusr/kernel/tests/fp32_honesty_regression/*.bin, shared y
                                 stored once) and its manifest's per-tree baseline flags
  jac_sample.npz                 the reference's reverse-AD Jacobian samples
                                 (experiments/revad_v5/jac_sample_fixed.jsonl)
  metric_scipy.npz               reference ScipyPop fits of a 256-tree stratified sample of
                                 the headline metric population at its full N (--metric)
  fd_pop1000.npz                 the reference FD variant's outputs on the pop.bin fixture
                                 (--fd)
  configs_full_scipy.npz         reference ScipyPop fits of 32-tree samples of the mid,
                                 physics, long and scale configurations at their own N
                                 (--configs-full; inputs stored as a digest)
  sharded_scipy.npz              reference ScipyPop fits of an 8-tree sample of the
                                 sample-sharded configuration at its own N = 10,000,000
                                 (--sharded; inputs stored as a digest)
The tests read only these files; the reference is not needed at test time.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _reference() -> Path:
    """The reference checkout, from CUSR_REFERENCE (required: there is no default path)."""
    ref = os.environ.get("CUSR_REFERENCE")
    if not ref or not (Path(ref) / "cusr" / "benchmark").is_dir():
        sys.exit("set CUSR_REFERENCE to the reference (TensorConv/CuSR) checkout")
    return Path(ref)


def pop_digest(pop: dict) -> str:
    """sha256 over the population arrays (bytecode, metas, c_init, inputs, targets)."""
    import hashlib

    h = hashlib.sha256()
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        h.update(np.ascontiguousarray(pop[k]).tobytes())
    return h.hexdigest()


def _pop_arrays(prefix: str, pop: dict) -> dict:
    out = {}
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        out[f"{prefix}/{k}"] = np.asarray(pop[k])
    for k in ("M", "total_nodes", "total_c", "N", "n_vars", "K_max", "max_stack"):
        out[f"{prefix}/{k}"] = np.asarray(int(pop[k]))
    return out


# (config, trees, samples) of the configs_scipy.npz samples: every configuration of the
# benchmark grammar at a size the reference's CPU fit finishes in seconds
CONFIG_SAMPLES = (("mid", 64, 1000), ("physics", 64, 1000), ("long", 64, 512), ("scale", 64, 1000))


def make_config_samples() -> None:
    """configs_scipy.npz: reference ScipyPop fits of sampled configurations."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from cusr.benchmark import backends, interp  # reference code

    from cusr_b200 import synth

    arr = {}
    for name, M, N in CONFIG_SAMPLES:
        pop = synth.make_config(name, M=M, N=N, seed=7)
        ref_pop = _as_ref(pop)
        sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(ref_pop)
        arr.update(_pop_arrays(name, pop))
        arr[f"{name}/scipy/c_final"] = sc.c_final
        arr[f"{name}/scipy/status"] = sc.status
        arr[f"{name}/scipy/loss64"] = interp.loss_pop(ref_pop, sc.c_final)
        arr[f"{name}/init/loss64"] = interp.loss_pop(ref_pop, pop["c_init"].astype(np.float64))
        print(name, "fitted", flush=True)
    np.savez_compressed(HERE / "configs_scipy.npz", **arr)


# stratified sample of the headline metric population (16,384 trees, seed 0) at its full
# N = 10,000: the trees behind the benchmarked fits/s, fitted by the reference's CPU backend
METRIC_SAMPLE = 256


def metric_sample_index(M: int = 16384, n: int = METRIC_SAMPLE) -> np.ndarray:
    """Tree indices of the metric sample: evenly spaced over the population."""
    return np.unique(np.linspace(0, M - 1, n).astype(np.int64))


def make_metric_sample() -> None:
    """metric_scipy.npz: reference ScipyPop fits of 256 trees of the metric population
    (synth 'metric', seed 0, N = 10,000, shared target row)."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from cusr.benchmark import backends, interp  # reference code

    from cusr_b200 import popio, synth

    full = synth.make_config("metric", seed=0)
    idx = metric_sample_index(int(full["M"]))
    pop = popio.slice_pop(full, idx)
    ref_pop = _as_ref(pop)
    sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(ref_pop)
    arr = _pop_arrays("pop", pop)
    arr.update({"index": idx, "scipy/c_final": sc.c_final, "scipy/status": sc.status,
                "scipy/nfev": sc.n_iter, "scipy/loss64": interp.loss_pop(ref_pop, sc.c_final),
                "init/loss64": interp.loss_pop(ref_pop, pop["c_init"].astype(np.float64))})
    np.savez_compressed(HERE / "metric_scipy.npz", **arr)


# (config, trees) of configs_full_scipy.npz: 32-tree samples of the configurations at their
# own N (mid 10,000; physics 100,000; long 4,096; scale 20,000)
CONFIG_SAMPLES_FULL = (("mid", 32), ("physics", 32), ("long", 32), ("scale", 32))


def make_config_samples_full() -> None:
    """configs_full_scipy.npz: reference ScipyPop fits of sampled configurations at full N."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from cusr.benchmark import backends, interp  # reference code

    from cusr_b200 import synth

    arr = {}
    for name, M in CONFIG_SAMPLES_FULL:
        pop = synth.make_config(name, M=M, seed=11)
        ref_pop = _as_ref(pop)
        sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(ref_pop)
        # the inputs and targets are large at full N: stored as a digest, the tests regenerate
        # them with cusr_b200.synth (seeded) and check the digest
        arr.update({k: v for k, v in _pop_arrays(name, pop).items()
                    if not k.endswith(("/xs", "/ym"))})
        arr[f"{name}/digest"] = np.asarray(pop_digest(pop))
        arr[f"{name}/scipy/c_final"] = sc.c_final
        arr[f"{name}/scipy/status"] = sc.status
        arr[f"{name}/scipy/loss64"] = interp.loss_pop(ref_pop, sc.c_final)
        arr[f"{name}/init/loss64"] = interp.loss_pop(ref_pop, pop["c_init"].astype(np.float64))
        print(name, "fitted", flush=True)
    np.savez_compressed(HERE / "configs_full_scipy.npz", **arr)


# trees of sharded_scipy.npz: the sample-sharded configuration at N = 10^7, where one
# reference fit takes minutes per core
SHARDED_SAMPLE = 8


def make_sharded_sample() -> None:
    """sharded_scipy.npz: reference ScipyPop fits of the sample-sharded configuration's
    grammar at its full N (10^7 samples), inputs stored as a digest."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from cusr.benchmark import backends, interp  # reference code

    from cusr_b200 import synth

    pop = synth.make_config("sharded", M=SHARDED_SAMPLE, seed=11)
    ref_pop = _as_ref(pop)
    sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(ref_pop)
    arr = {k: v for k, v in _pop_arrays("sharded", pop).items()
           if not k.endswith(("/xs", "/ym"))}
    arr["sharded/digest"] = np.asarray(pop_digest(pop))
    arr["sharded/scipy/c_final"] = sc.c_final
    arr["sharded/scipy/status"] = sc.status
    arr["sharded/scipy/loss64"] = interp.loss_pop(ref_pop, sc.c_final)
    arr["sharded/init/loss64"] = interp.loss_pop(ref_pop, pop["c_init"].astype(np.float64))
    np.savez_compressed(HERE / "sharded_scipy.npz", **arr)


def make_fd_golden() -> None:
    """fd_pop1000.npz: the reference FD variant's outputs on its pop.bin fixture
    (cusr/kernel/tests/golden/fd/pop1000: status, c_final; 50 iterations,
    tests/test_inproc_parity.py:44) and their fp64 losses."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    from cusr.benchmark import interp, popio  # reference code

    pop = popio.load_pop_bin(REF / "data" / "fixtures" / "pop.bin")
    gd = REF / "cusr" / "kernel" / "tests" / "golden" / "fd" / "pop1000"
    c = np.fromfile(gd / "c_final.bin", np.float32)
    st = np.fromfile(gd / "status.bin", np.int32)
    np.savez_compressed(HERE / "fd_pop1000.npz", status=st, c_final=c,
                        loss64=interp.loss_pop(pop, c.astype(np.float64)))


def make_honesty() -> None:
    """fp32_honesty.npz: the fp32-honesty regression fixtures of the reference."""
    REF = _reference()
    sys.path.insert(0, str(REF))
    from cusr.benchmark import popio  # reference loader

    d = REF / "cusr" / "kernel" / "tests" / "fp32_honesty_regression"
    manifest = json.loads((d / "manifest.json").read_text())
    arr = {"names": np.asarray(sorted(manifest["fixtures"]))}
    for i, name in enumerate(sorted(manifest["fixtures"])):
        fx = manifest["fixtures"][name]
        pop = popio.load_pop_bin(d / fx["file"])
        pop = {k: pop[k] for k in pop}
        ym = np.asarray(pop["ym"], np.float32).reshape(int(pop["M"]), int(pop["N"]))
        assert np.all(ym == ym[0]), name          # every fixture shares one target row
        pop["ym"] = ym[0]
        arr.update(_pop_arrays(f"f{i}", pop))
        arr[f"f{i}/fd_serious"] = np.asarray([t["fd"]["serious"] for t in fx["trees"]])
        arr[f"f{i}/ad_serious"] = np.asarray([t["ad"]["serious"] for t in fx["trees"]])
    np.savez_compressed(HERE / "fp32_honesty.npz", **arr)


def main() -> None:
    if "--configs" in sys.argv:
        make_config_samples()
        return
    if "--honesty" in sys.argv:
        make_honesty()
        return
    if "--metric" in sys.argv:
        make_metric_sample()
        return
    if "--fd" in sys.argv:
        make_fd_golden()
        return
    if "--configs-full" in sys.argv:
        make_config_samples_full()
        return
    if "--sharded" in sys.argv:
        make_sharded_sample()
        return
    REF = _reference()
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from cusr.benchmark import backends, interp, popio  # reference code

    from cusr_b200 import synth

    kt = REF / "cusr" / "kernel" / "tests"
    # ---- known-answer fixtures ----
    arrays, truths = {}, {}
    names = ["pop_fixture", "pop_fixture_op", "pop_fixture_stress", "pop_fixture_scale_1e-6",
             "pop_fixture_scale_1e-3", "pop_fixture_scale_1e0", "pop_fixture_scale_1e3",
             "pop_fixture_scale_1e6"]
    for name in names:
        pop = popio.load_pop_bin(kt / f"{name}.bin")
        arrays.update(_pop_arrays(name, pop))
        # reference fp64 loss at c_init
        arrays[f"{name}/loss_init64"] = interp.loss_pop(pop, pop["c_init"].astype(np.float64))
    for tj in ("pop_fixture_truth.json", "pop_fixture_op_truth.json",
               "pop_fixture_stress_truth.json", "pop_fixture_scale_truth.json"):
        truths[tj] = json.loads((kt / tj).read_text())
    np.savez_compressed(HERE / "fixtures.npz", **arrays)
    (HERE / "fixtures.json").write_text(json.dumps(truths, indent=1))

    # ---- pop1000 + reference kernel goldens + reference scipy fits ----
    pop = popio.load_pop_bin(REF / "data" / "fixtures" / "pop.bin")
    assert np.all(pop["ym"] == pop["ym"][0])
    gd = kt / "golden" / "ad" / "pop1000"
    g_c = np.fromfile(gd / "c_final.bin", np.float32)
    g_st = np.fromfile(gd / "status.bin", np.int32)
    g_li = np.fromfile(gd / "loss_init.bin", np.float32)
    g_lf = np.fromfile(gd / "loss_final.bin", np.float32)
    sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(pop)
    arr = _pop_arrays("pop", pop)
    arr["pop/ym"] = pop["ym"][0].copy()            # shared row
    arr.update({
        "refkernel/c_final": g_c, "refkernel/status": g_st,
        "refkernel/loss_init": g_li, "refkernel/loss_final": g_lf,
        "refkernel/loss64": interp.loss_pop(pop, g_c.astype(np.float64)),
        "init/loss64": interp.loss_pop(pop, pop["c_init"].astype(np.float64)),
        "scipy/c_final": sc.c_final, "scipy/status": sc.status, "scipy/nfev": sc.n_iter,
        "scipy/loss64": interp.loss_pop(pop, sc.c_final),
    })
    np.savez_compressed(HERE / "pop1000.npz", **arr)

    # ---- interpreter vectors ----
    pr1 = synth.make_config("pr1", M=64, N=200, seed=0)
    vals = np.stack([interp.eval_pop_tree(_as_ref(pr1), m,
                                          pr1["c_init"][pr1["metas"][m][2]:
                                                        pr1["metas"][m][2] + pr1["metas"][m][3]])
                     for m in range(pr1["M"])])
    p1000 = {k: pop[k] for k in pop}
    v1000 = np.stack([interp.eval_pop_tree(p1000, m,
                                           pop["c_init"][pop["metas"][m][2]:
                                                         pop["metas"][m][2] + pop["metas"][m][3]])
                      for m in range(64)])
    iv = _pop_arrays("pr1", pr1)
    iv["pr1/values"] = vals
    iv["pop1000/values"] = v1000
    np.savez_compressed(HERE / "interp_vectors.npz", **iv)

    # ---- PR1 configuration: reference scipy fits ----
    pr1 = synth.make_config("pr1", seed=0)
    ref_pop = _as_ref(pr1)
    sc = backends.ScipyPop(nproc=os.cpu_count()).fit_pop(ref_pop)
    arr = _pop_arrays("pop", pr1)
    arr.update({"scipy/c_final": sc.c_final, "scipy/status": sc.status,
                "scipy/nfev": sc.n_iter, "scipy/loss64": interp.loss_pop(ref_pop, sc.c_final),
                "init/loss64": interp.loss_pop(ref_pop, pr1["c_init"].astype(np.float64))})
    np.savez_compressed(HERE / "pr1_scipy.npz", **arr)

    # ---- reference reverse-AD Jacobian samples ----
    rows = [json.loads(l) for l in
            (REF / "experiments" / "revad_v5" / "jac_sample_fixed.jsonl").read_text().splitlines()
            if l.strip()]
    js = {"n": np.asarray(len(rows))}
    for i, r in enumerate(rows):
        js[f"{i}/nt"] = np.asarray(r["nt"], np.int32)
        js[f"{i}/nv"] = np.asarray(r["nv"], np.float32)
        js[f"{i}/ci"] = np.asarray(r["ci"], np.int32)
        js[f"{i}/c"] = np.asarray(r["c"], np.float32)
        js[f"{i}/n_vars"] = np.asarray(int(r["n_vars"]))
        js[f"{i}/x"] = np.asarray([p["x"] for p in r["pts"]], np.float32)
        js[f"{i}/rev"] = np.asarray([p["rev"] for p in r["pts"]], np.float64)
        js[f"{i}/fwd"] = np.asarray([p["fwd"] for p in r["pts"]], np.float64)
    np.savez_compressed(HERE / "jac_sample.npz", **js)
    print("golden fixtures written to", HERE)


def _as_ref(pop: dict) -> dict:
    """The reference loader's pop layout: ym is [M, N] (a shared row is replicated)."""
    out = dict(pop)
    ym = np.asarray(pop["ym"], np.float32)
    if ym.ndim == 1:
        out["ym"] = np.ascontiguousarray(np.broadcast_to(ym, (int(pop["M"]), int(pop["N"]))))
    return out


if __name__ == "__main__":
    main()
