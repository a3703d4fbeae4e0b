"""Benchmark: LM fits/s of the batched constant-fitting engine (cusr_b200) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step" = one complete LM fit of the population): the headline configuration
"pop 16k, N=10k, 50 iters" — 16,384 random expression trees (bytecode length 7-63, operators
+ - * / sin cos exp log|.| sqrt|.|, 5 input variables x ~ U[-5,5], K ~ U{1..12} unpadded),
N = 10,000 samples, one shared target row (a ground-truth tree + N(0, 0.05^2) noise), fp32,
50 LM iterations. Synthetic and seeded (the reference publishes no dataset for this metric).

Multi-GPU (torchrun, one rank per GPU): weak scaling — the global population has 16,384 trees
per GPU and is split into cost-balanced shards (LPT); ranks fit their shards with no exchange
and the time is the max over ranks. Results are gathered to rank 0 once, outside the timing.

`value`: fits/s with the population already resident in HBM (co_load once, then co_fit_loaded
per step), device-timed with CUDA events on the engine's stream. `e2e`: the same metric through
the public extended entry point (co_optimize_ex) from pinned host buffers, H2D and D2H inside.
`--impl reference`: the reference's CPU path (ScipyPop restated in oracle/scipy_lm.py:
scipy least_squares LM per tree, one process per host core) on a bounded sample of trees; its
line also carries `reference_gpu`, the reference's own CUDA LM path (batch_lm_revad built from
its sources for sm_100a by oracle/Makefile) timed on the same 16,384-tree population, when that
binary is present. `--impl reference_gpu` prints that measurement as its own line, and the
default arm (one GPU) carries it as `vs_reference_gpu` {ours, ref, ratio}.

Reports that are files (the nvidia-smi clock samples) go to --out-dir, default
$CUSR_REPORT_DIR, else a temporary directory.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "LM fits/sec (pop 16k, N=10k, 50 iters) at 1/8 GPU; node-evals/s vs roofline"
CONFIG = "metric"
M_PER_GPU = 16384
PEAKS = ROOT / "MEASURED_PEAKS.json"
PROFILE_SUMMARY = ROOT / "profiles" / "lm_eval_kernel_metric.md"
INST_SUMMARY = ROOT / "profiles" / "lm_eval_kernel_sfu_vs_ieee_instructions.md"
L2_BYTES = 126 << 20     # B200 L2
CPU_BASELINE_MAX_N = 1_000_000   # larger N: a single scipy fit outlasts the bounded sample


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


class ClockSampler:
    """nvidia-smi clock / throttle samples of this rank's GPU during the timed region."""

    def __init__(self, gpu: int, out: Path):
        self.out = out
        self.proc = None
        try:
            self.f = open(out, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu), "--query-gpu=index,clocks.sm,clocks.max.sm,"
                 "power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_population(world: int):
    from cusr_b200 import synth

    return synth.make_config(CONFIG, M=M_PER_GPU * world, seed=0)


def pinned_copy(pop: dict) -> dict:
    """Host copy of the pop's arrays in page-locked memory (the e2e inputs)."""
    import torch

    out = dict(pop)
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        a = np.ascontiguousarray(pop[k])
        t = torch.empty(a.shape, dtype=getattr(torch, a.dtype.name), pin_memory=True)
        t.numpy()[...] = a
        out[k] = t.numpy()
    return out


def out_dir(args) -> Path:
    d = args.out_dir or os.environ.get("CUSR_REPORT_DIR") or tempfile.mkdtemp(prefix="cusr_bench_")
    p = Path(d)
    p.mkdir(parents=True, exist_ok=True)
    return p


def profile_value(key: str, summary: Path = PROFILE_SUMMARY):
    """A figure recorded in a committed ncu summary (default profiles/lm_eval_kernel_metric.md,
    lines `key: value`): NOT measured by this run, so it is returned with its source and the
    commit it was captured at."""
    if not summary.exists():
        return None
    val, commit = None, None
    for line in summary.read_text().splitlines():
        t = line.strip()
        if t.startswith(key + ":"):
            try:
                val = float(t.split(":", 1)[1].strip().split()[0])
            except ValueError:
                val = None
        elif t.startswith("captured_at:"):
            commit = t.split(":", 1)[1].strip()
    if val is None:
        return None
    return {"value": val, "source": str(summary.relative_to(ROOT)),
            "captured_at": commit, "measured_in_this_run": False}


def issue_estimate(node_evals: float, eval_ms: float, clk: dict):
    """Issue-slot fraction of the timed evaluation launches, estimated live: the committed
    capture's thread-instructions per node-eval (a per-workload constant of the interpreter)
    x this run's node-evals / eval time, over the issue peak 148 SMs x 4 schedulers x the
    sampled SM clock x 32 threads."""
    ipn = profile_value("thread_instructions_per_node_eval", INST_SUMMARY)
    mhz = clk.get("sm_mhz") if isinstance(clk, dict) else None
    if not ipn or not mhz or eval_ms <= 0:
        return None
    try:
        import torch

        sms = torch.cuda.get_device_properties(0).multi_processor_count
    except Exception:  # noqa: BLE001
        sms = 148
    peak = sms * 4 * mhz * 1e6 * 32
    rate = ipn["value"] * node_evals / (eval_ms / 1e3)
    return {"frac": rate / peak, "thread_inst_per_s": rate, "peak_thread_inst_per_s": peak,
            "inst_per_node_eval": ipn}


def measured_hbm_peak():
    """(GB/s, source) of the copy bandwidth in MEASURED_PEAKS.json (driver-measured on this
    pool's B200s), else the pool's earlier measurement (6,650 GB/s, "fallback")."""
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback (earlier measurement on this pool)"


def config_roofline(st_sum: dict, pop: dict, precision: str, fp_peaks: tuple) -> dict:
    """Live roofline of the evaluation kernel over a configuration's timed fits, from the
    engine's own counters (summed over the timed steps): FLOPs of the interpreter and
    normal equations (2 per operator node + 2 per block entry, per evaluated tree-sample)
    over its device time, against the in-run FMA probe peak of the fit's precision; for
    per-tree targets (a target row per tree, streamed from HBM every pass) also the target
    bytes (4 per evaluated tree-sample) over the same time, against the measured copy
    bandwidth. `bound` is the roof with the larger fraction."""
    eval_s = st_sum["eval_ms"] / 1e3
    if eval_s <= 0:
        return {"unavailable": "no evaluation time recorded"}
    fp64 = precision == "fp64"
    peak = fp_peaks[1] if fp64 else fp_peaks[0]
    tf = st_sum["flops"] / eval_s / 1e12
    fp = {"bound": "fp64" if fp64 else "fp32", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
          "frac": tf / peak if peak else None,
          "peak_source": "measured FMA probe (co_probe_peak, same run)"}
    out = {"kernel": "lm_eval_kernel", "fp": fp, "eval_ms": st_sum["eval_ms"],
           "avg_launch_ms": st_sum["eval_ms"] / max(1, st_sum["eval_launches"]),
           "node_evals_per_s_eval": st_sum["node_evals"] / eval_s}
    ym = np.asarray(pop["ym"])
    per_tree_y = ym.ndim == 2 and ym.shape[0] > 1
    N, n_vars = int(pop["N"]), int(pop["n_vars"])
    x_in_l2 = 4 * N * (n_vars + 1) <= L2_BYTES
    if per_tree_y or not x_in_l2:
        per_sample = (4 if per_tree_y else 0) + (0 if x_in_l2 else 4 * (n_vars + (0 if per_tree_y else 1)))
        gbs = per_sample * st_sum["sample_evals"] / eval_s / 1e9
        hpk, src = measured_hbm_peak()
        what = ("the tree's target" if per_tree_y else "") + \
               ("" if x_in_l2 else (" and " if per_tree_y else "") + "the sample's inputs" +
                ("" if per_tree_y else " and shared target"))
        out["hbm"] = {"bound": "hbm", "achieved": gbs, "peak": hpk, "unit": "GB/s",
                      "frac": gbs / hpk, "peak_source": src,
                      "bytes_def": f"{per_sample} B per evaluated (tree, sample): {what} "
                                   f"({'X is L2-resident' if x_in_l2 else 'X and y exceed L2'})"}
    else:
        out["hbm_note"] = "one shared target row and X are L2-resident: no HBM stream per pass"
    best = max((r for r in (fp, out.get("hbm")) if r and r.get("frac") is not None),
               key=lambda r: r["frac"], default=fp)
    out.update(bound=best["bound"], achieved=best["achieved"], peak=best["peak"],
               unit=best["unit"], frac=best["frac"])
    return out


def cpu_baseline(pop: dict, target_s: float = 15.0) -> dict:
    """ScipyPop restatement on all host cores, on a stratified sample of the trees sized to
    about `target_s` seconds of fitting (pool start-up excluded, as the reference's
    persistent pool)."""
    from oracle import scipy_lm

    M = int(pop["M"])
    cores = os.cpu_count() or 1
    with scipy_lm.Pool(cores) as pool:
        pool.warm()
        calib = np.linspace(0, M - 1, min(M, 2 * cores)).astype(np.int64)
        r0 = pool.fit_pop(pop, trees=calib)
        rate = len(calib) / max(r0["wall"], 1e-3)
        n = int(min(M, max(2 * cores, rate * target_s)))
        idx = np.unique(np.linspace(0, M - 1, n).astype(np.int64))
        res = pool.fit_pop(pop, trees=idx)
    wall = res["wall"]
    return {"value": len(idx) / wall, "unit": "fits/s", "cores": cores, "kind": "port",
            "sample": f"{len(idx)} of {M} trees (stratified), N={pop['N']}, scipy "
                      f"least_squares lm xtol=ftol=1e-10 max_nfev=200, fp64, {wall:.1f} s",
            "wall_s": wall}


def reference_gpu(pop: dict, runs: int = 3, warmup: int = 1) -> dict:
    """The reference's own CUDA LM path on `pop`: oracle/_ref/batch_lm_revad_prof (its sources
    built for sm_100a, fast-math fp32, host-driven loop, 50 iterations), timed by its own
    PROFILE_JSON loop_ms; trees/s = (M - K0 trees) / loop_ms, its convention
    (experiments/e6_kernel_sweep/sweep_e6.py:126-132). Median of `runs` runs after `warmup`."""
    from oracle import ref_gpu

    try:
        with ref_gpu.RefGPU(pop) as rg:
            for _ in range(warmup):
                rg.run(max_iter=50)
            outs = [rg.run(max_iter=50) for _ in range(runs)]
            n_nodes = int(np.asarray(rg.pop["metas"])[:, 1].sum())
    except (FileNotFoundError, ValueError, RuntimeError, subprocess.TimeoutExpired) as e:
        return {"unavailable": str(e)[:300]}
    loops = sorted(o["loop_ms"] for o in outs)
    med = loops[len(loops) // 2]
    last = outs[-1]
    M = int(pop["M"])
    return {"value": (M - int(np.sum(np.asarray(pop["metas"])[:, 3] == 0))) / (med / 1e3),
            "unit": "fits/s", "loop_ms_runs": loops, "loop_ms": med,
            "iters_run": int(last["profile"]["iters_run"]),
            "total_ms": float(last["profile"]["total_ms"]),
            "statuses": np.bincount(last["status"], minlength=5).tolist(),
            "binary": "oracle/_ref/batch_lm_revad_prof: cusr/kernel/batch_lm_revad.cu built for "
                      "sm_100a with the reference's flags (-O2 --use_fast_math) and -DPROFILE",
            "population": f"the same {M} trees (metric config, seed 0); log|x| and sqrt|x| "
                          f"encoded as LOG(ABS(x)) / SQRT(ABS(x)) ({n_nodes} nodes)",
            "convention": "trees/s = (M - K0) / loop_ms (LM loop only, setup and load excluded)"}


def run_reference_gpu(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    pop = make_population(1)
    rg = reference_gpu(pop, runs=max(1, min(args.steps, 5)), warmup=max(1, min(args.warmup, 2)))
    line = {"impl": "reference_gpu", "metric": METRIC, "value": rg.get("value"),
            "unit": "fits/s", "n_gpus": 1, "steps": len(rg.get("loop_ms_runs", [])),
            "warmup": max(1, min(args.warmup, 2)),
            "ms_per_step": rg.get("loop_ms"), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "pop 16k, N=10k, 50 iters (metric config, seed 0)"},
            "reference_gpu": rg}
    print(json.dumps(line), flush=True)


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    pop = make_population(1)
    from oracle import scipy_lm

    cores = os.cpu_count() or 1
    M = int(pop["M"])
    rng = np.random.default_rng(1)
    with scipy_lm.Pool(cores) as pool:
        pool.warm()
        calib = pool.fit_pop(pop, trees=rng.choice(M, min(M, 2 * cores), replace=False))
        rate = calib["n_fitted"] / max(calib["wall"], 1e-3)
        # each step about 20 s of fitting, so the whole run stays within a few minutes
        per_step = int(min(M, max(2 * cores, rate * 20.0)))
        for _ in range(args.warmup):
            pool.fit_pop(pop, trees=rng.choice(M, min(M, cores), replace=False))
        times = []
        for _ in range(args.steps):
            idx = np.sort(rng.choice(M, per_step, replace=False))
            times.append(pool.fit_pop(pop, trees=idx)["wall"])
    value = per_step * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "fits/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "pop 16k, N=10k, 50 iters (metric config, seed 0)",
                   "sample_per_step": f"{per_step} random trees of the 16,384", "N": pop["N"]},
        "cpu_baseline": {"value": value, "unit": "fits/s", "cores": cores, "kind": "port",
                         "sample": f"{per_step} trees per step, scipy least_squares lm, "
                                   f"one process per core"},
        "e2e": {"value": value, "unit": "fits/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if not args.no_reference_gpu:
        line["reference_gpu"] = reference_gpu(pop)
    print(json.dumps(line), flush=True)


def metric_scipy_sample():
    """The 256-tree stratified sample of the metric population at N = 10,000 and the
    reference's scipy fp64 losses of it (tests/golden/metric_scipy.npz, made by the
    reference's ScipyPop); (None, None) when the fixture is absent."""
    golden = ROOT / "tests" / "golden" / "metric_scipy.npz"
    if not golden.exists():
        return None, None
    z = np.load(golden)
    sample = {k: z[f"pop/{k}"] for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym")}
    sample.update({k: int(z[f"pop/{k}"]) for k in ("M", "total_nodes", "total_c", "N",
                                                    "n_vars", "K_max", "max_stack")})
    return sample, z["scipy/loss64"]


def north_star_fraction(co, sample: dict, ref: np.ndarray, c_final) -> float:
    """Fraction of the sample's trees (K > 0, finite scipy loss) whose fp64 loss at c_final is
    within 1e-6 relative of, or below, the reference scipy fit's."""
    blk = co.evaluate(sample, c=c_final, precision="fp64", values=False, blocks=True)["blocks"]
    l64 = np.array([b[-1] for b in blk])
    elig = (np.asarray(sample["metas"])[:, 3] > 0) & np.isfinite(ref)
    return float(np.mean((l64 <= ref * (1 + 1e-6) + 1e-12)[elig]))


def headline_parity(co) -> dict | None:
    """The north-star fraction of the mode `value` times (one start, the reference LM, 50
    iterations, fp32) and of its fp32_fast numerics, on the metric scipy sample: the fit
    quality behind the headline fits/s, reported beside it."""
    sample, ref = metric_scipy_sample()
    if sample is None:
        return None
    out = {"sample": f"{int(sample['M'])} trees of the metric population (stratified), "
                     f"N={int(sample['N'])}, reference scipy lm xtol=ftol=1e-10 max_nfev=200",
           "criterion": "fp64 loss within 1e-6 relative of, or below, the scipy fit"}
    for prec in ("fp32", "fp32_fast"):
        r = co.optimize_ex(sample, max_iter=50, precision=prec)
        out[f"within_1e-6_or_better_{prec}"] = north_star_fraction(co, sample, ref,
                                                                   r["c_final"])
    # the same fraction for the reference's own CUDA path (the vs_reference_gpu binary) on the
    # same sample: the quality of the fit the headline mode replaces
    from oracle import ref_gpu

    try:
        with ref_gpu.RefGPU(sample) as rg:
            c_ref = rg.run(max_iter=50)["c_final"]
        out["within_1e-6_or_better_reference_gpu"] = north_star_fraction(co, sample, ref, c_ref)
    except (FileNotFoundError, ValueError, RuntimeError, subprocess.TimeoutExpired) as e:
        out["reference_gpu_unavailable"] = str(e)[:300]
    out["parity_grade_mode"] = "parity_mode (same sample, multi-start + fp64 polish)"
    return out


def parity_mode(co, pop: dict) -> dict:
    """The parity-grade fit (cusr_b200.multistart defaults, co_inproc.PARITY: 128 trust-region
    starts per tree explored in fp32 on the device, two waves, fp64 polish from 8 starts
    around each tree's best): fits/s on a
    2,048-tree stratified slice of the metric population (device time of the multi-start call
    plus the polish call), and the north-star fraction — fp64 loss within 1e-6 of, or better
    than, the reference scipy fit — on the 256-tree scipy sample of the same population
    (tests/golden/metric_scipy.npz, made by the reference's ScipyPop). `fast`: the same for
    co_inproc.PARITY_FAST (single-start polish)."""
    from cusr_b200 import co_inproc, multistart, popio

    sub = popio.slice_pop(pop, np.unique(np.linspace(0, int(pop["M"]) - 1, 2048).astype(np.int64)))
    sample, ref = metric_scipy_sample()

    def measure(kw: dict) -> dict:
        multistart.fit_multistart(co, popio.slice_pop(sub, 64), **kw)            # warm-up
        res = multistart.fit_multistart(co, sub, **kw)
        st = res["stats"]
        ms = st["device_ms"] + co.stats()["device_ms"]
        frac = None
        if sample is not None:
            r = multistart.fit_multistart(co, sample, **kw)
            frac = north_star_fraction(co, sample, ref, r["c_final"])
        return {"value": int(sub["M"]) / (ms / 1e3), "unit": "fits/s",
                "within_1e-6_or_better": frac, "starts": int(st["n_starts"]),
                "fits_run": int(st["fits_run"]), "trees_retired": int(st["trees_retired"]),
                "trees": int(sub["M"]), "device_ms": ms}

    out = measure(multistart.preset_kwargs(co_inproc.PARITY))
    out.update(dtype="f32 starts, f64 polish", note="the parity-grade mode (co_inproc.PARITY: "
               "128 device-side trust-region starts explored in fp32, then each tree's best "
               "polished in fp64 from 8 starts around it) on a 2,048-tree slice of the metric "
               "population; the fraction on the 256-tree reference scipy sample of that "
               "population")
    fast = measure(multistart.preset_kwargs(co_inproc.PARITY_FAST))
    fast.update(dtype="f32 starts, f64 polish", note="co_inproc.PARITY_FAST: the same with a "
                "single-start fp64 polish")
    out["fast"] = fast
    top = measure(multistart.preset_kwargs(co_inproc.PARITY_MAX))
    top.update(dtype="f32 starts, f64 polish, dd-f64 starts", note="co_inproc.PARITY_MAX: "
               "PARITY and 16 fp64 trust-region starts from c_init on double-double normal "
               "equations")
    out["max"] = top
    return out


def run_ours(args, world: int, rank: int, local: int) -> None:
    from cusr_b200 import InProcessCO, shard

    pop = make_population(world)
    if world > 1:
        mine, idx = shard.shard(pop, rank, world)
    else:
        mine, idx = pop, np.arange(int(pop["M"]))
    co = InProcessCO(device_id=local if world > 1 else 0)
    fp32_peak, fp64_peak = co.probe_peak()
    co.load(mine, precision="fp32", y_shared=True)
    for _ in range(args.warmup):
        co.fit_loaded(max_iter=50)
    barrier(world)
    clocks = ClockSampler(local if world > 1 else 0, out_dir(args) / f"clocks_rank{rank}.csv")
    dev_ms, eval_ms, eval_launches, launches, flops, node_evals = [], 0.0, 0, 0, 0.0, 0
    res = None
    for _ in range(args.steps):
        res = co.fit_loaded(max_iter=50)
        st = co.stats()
        dev_ms.append(st["device_ms"])
        eval_ms += st["eval_ms"]
        eval_launches += st["eval_launches"]
        launches += st["kernel_launches"]
        flops += st["flops"]
        node_evals += st["node_evals"]
    clk = clocks.stop()
    barrier(world)
    total_ms = max_over_ranks(float(sum(dev_ms)), world)

    # the same fits with the reference kernel's numerics (--use_fast_math instantiation)
    for _ in range(args.warmup):
        co.fit_loaded(max_iter=50, precision="fp32_fast")
    barrier(world)
    fast_ms = 0.0
    for _ in range(args.steps):
        co.fit_loaded(max_iter=50, precision="fp32_fast")
        fast_ms += co.stats()["device_ms"]
    barrier(world)
    fast_ms = max_over_ranks(fast_ms, world)
    M_total = int(pop["M"])
    value = M_total * args.steps / (total_ms / 1e3)
    node_evals_total = sum_over_ranks(float(node_evals), world)

    # e2e through the public extended entry point, pinned host buffers
    host = pinned_copy(mine)
    h2d = sum(np.asarray(host[k]).nbytes for k in ("nt", "nv", "ci", "metas", "c_init", "xs"))
    h2d += int(mine["N"]) * 4
    d2h = int(mine["total_c"]) * 8 + int(mine["M"]) * (4 + 8 + 8 + 4)
    import torch

    torch.cuda.set_device(local if world > 1 else 0)
    co.optimize_ex(host, max_iter=50, precision="fp32", y_shared=True)   # warm
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        co.optimize_ex(host, max_iter=50, precision="fp32", y_shared=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = M_total * args.steps / (e2e_ms / 1e3)

    # gather the fits of the last timed step to rank 0 (outside the timing)
    if world > 1:
        shard.gather_to_root(pop, idx, res)

    if rank != 0:
        return
    avg_launch_ms = eval_ms / max(1, eval_launches)
    achieved = flops / (eval_ms / 1e3) / 1e12 if eval_ms > 0 else None
    roofline = {
        "bound": "fp32", "kernel": "lm_eval_kernel", "unit": "TFLOP/s",
        "achieved": achieved, "peak": fp32_peak,
        "frac": (achieved / fp32_peak) if achieved and fp32_peak else None,
        "peak_source": "measured FP32 FMA probe (co_probe_peak, same run); MEASURED_PEAKS.json "
                       "holds only HBM and bf16 tensor peaks",
        "traffic": (profile_value("traffic_bytes_per_launch") or {}).get("value"),
        "traffic_source": profile_value("traffic_bytes_per_launch"),
        "traffic_note": "dram read+write bytes of one evaluation launch from the committed ncu "
                        "capture (not measured in this run); inputs and partial sums are "
                        "L2-resident",
        "issue": {"bound": "issue", "achieved_pct": profile_value("issue_active_pct"),
                  "note": "issue slots busy on the evaluation kernel, from the committed ncu "
                          "capture (not measured in this run): the interpreter is bound by "
                          "instruction issue, not FMA or HBM throughput",
                  "live_estimate": issue_estimate(float(node_evals), eval_ms, clk)},
        "avg_launch_ms": avg_launch_ms,
        "flops_def": "per evaluated (tree, sample): 2 per operator node (value + adjoint) + "
                     "2 per normal-equation entry (K+1)(K+2)/2",
        "node_evals_per_s": node_evals_total / (total_ms / 1e3),
        "fp64_peak_tflops": fp64_peak,
    }
    line = {
        "metric": METRIC, "value": value, "unit": "fits/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "pop 16k per GPU, N=10k, 50 iters (metric config, seed 0)",
                   "trees": M_total, "N": int(pop["N"]), "max_iter": 50,
                   "parallelism": f"expression-sharded x{world} (LPT cost-balanced)",
                   "l2": "inputs resident (X 200 KB, y 40 KB) — the kernel is compute bound; "
                         "no L2 flush between steps"},
        "e2e": {"value": e2e_value, "unit": "fits/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "entry": "co_optimize_ex (pinned host buffers)"},
        "roofline": roofline,
        "fp32_fast": {"value": M_total * args.steps / (fast_ms / 1e3),
                      "ms_per_step": fast_ms / args.steps,
                      "note": "same fits, interpreter built with the reference kernel's "
                              "--use_fast_math flags (CO_PREC_FP32_FAST); measured after the "
                              "headline steps"},
        "gpu_launches": int(launches),
        "clocks": clk,
        "node_evals_per_s": roofline["node_evals_per_s"],
    }
    if world == 1 and not args.no_parity_mode:
        try:
            line["fit_parity"] = headline_parity(co)
        except Exception as e:  # noqa: BLE001 - a report field; the measured line stands
            line["fit_parity"] = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
        line["parity_mode"] = parity_mode(co, pop)
    if world == 1 and not args.no_reference_gpu:
        # the reference's own CUDA path on the same population and box (a subprocess of its
        # binary); its convention counts the LM loop only, as `value` does
        rg = reference_gpu(pop, runs=2, warmup=1)
        line["vs_reference_gpu"] = {
            "ours": line["value"], "ref": rg.get("value"),
            "ratio": (line["value"] / rg["value"]) if rg.get("value") else None,
            "same_population": True, "reference_gpu": rg}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(pop)
    print(json.dumps(line), flush=True)


def run_config(args, world: int = 1, rank: int = 0, local: int = 0) -> None:
    """One BASELINE configuration (pr1, mid, physics, long, scale, sharded): resident-input
    fits/s and node-evals/s, device-timed, with its CPU baseline sample. Under torchrun the
    configuration's population is split into cost-balanced expression shards, one per rank
    (strong scaling: the population is fixed), time = max over ranks."""
    from cusr_b200 import InProcessCO, shard, synth

    name = args.config
    pop = synth.make_config(name, M=args.M, N=args.N, seed=0)
    precision, max_iter = pop["precision"], int(pop["max_iter"])
    if args.fast_math and precision == "fp32":
        precision = "fp32_fast"
    shared = np.asarray(pop["ym"]).ndim == 1
    mine = shard.shard(pop, rank, world)[0] if world > 1 else pop
    co = InProcessCO(device_id=local if world > 1 else 0)
    peaks = co.probe_peak()
    co.load(mine, precision=precision, y_shared=shared)
    for _ in range(args.warmup):
        co.fit_loaded(max_iter=max_iter)
    barrier(world)
    clocks = ClockSampler(local if world > 1 else 0, out_dir(args) / f"clocks_{name}_rank{rank}.csv")
    dev, nodes, launches, res = [], 0, 0, None
    st_sum = dict.fromkeys(("eval_ms", "flops", "node_evals", "sample_evals", "eval_launches"), 0)
    for _ in range(args.steps):
        res = co.fit_loaded(max_iter=max_iter)
        st = co.stats()
        dev.append(st["device_ms"])
        nodes += st["node_evals"]
        launches += st["kernel_launches"]
        for k in st_sum:
            st_sum[k] += st[k]
    clk = clocks.stop()
    barrier(world)
    total_ms = max_over_ranks(float(sum(dev)), world)
    nodes = sum_over_ranks(float(nodes), world)
    if rank != 0:
        return
    M = int(pop["M"])
    line = {"metric": f"LM fits/sec ({name}: M={M}, N={pop['N']}, {max_iter} iters, {precision})",
            "value": M * args.steps / (total_ms / 1e3), "unit": "fits/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "f64" if precision == "fp64" else "f32", "data": "synthetic",
            "config": {"workload": name, "trees": M, "N": int(pop["N"]), "max_iter": max_iter,
                       "y_shared": bool(shared), "precision": precision},
            "node_evals_per_s": nodes / (total_ms / 1e3), "gpu_launches": launches,
            "statuses": np.bincount(res["status"], minlength=5).tolist(),
            "roofline": config_roofline(st_sum, mine, precision, peaks), "clocks": clk}
    if world > 1:
        line["config"]["parallelism"] = f"expression-sharded x{world} (LPT cost-balanced)"
    if not args.no_cpu_baseline and world == 1:
        if int(pop["N"]) > CPU_BASELINE_MAX_N:
            # one scipy fit over 10^7 samples takes about a minute per core: no bounded sample
            line["cpu_baseline"] = {"unavailable": f"N = {pop['N']}: one scipy fit per core "
                                                   "exceeds the bounded sample's time"}
        else:
            line["cpu_baseline"] = cpu_baseline(pop, target_s=10.0)
    print(json.dumps(line), flush=True)


def run_sample_sharded(args, world: int, rank: int, local: int) -> None:
    """The sample-sharded configuration (M=512 trees, N=10,000,000 samples, fp32, 30 iters)
    on `world` GPUs: every rank loads all trees and its contiguous slice of the samples; the
    engine all-reduces the per-tree normal equations over NCCL every iteration. Strong
    scaling (the problem is fixed); time = max over ranks of the device-timed fit."""
    from cusr_b200 import InProcessCO, co_inproc, shard, synth

    pop = synth.make_config("sharded", M=args.M, N=args.N, seed=0)
    precision, max_iter = pop["precision"], int(pop["max_iter"])
    mine = shard.sample_slice(pop, rank, world) if world > 1 else pop
    co = InProcessCO(device_id=local if world > 1 else 0)
    peaks = co.probe_peak()
    if world > 1:
        import torch.distributed as dist

        box = [co_inproc.shard_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        co.shard_init(box[0], world, rank, timeout_s=120.0)
    co.load(mine, precision=precision, y_shared=True)
    sharded = world > 1
    for _ in range(args.warmup):
        co.fit_loaded(max_iter=max_iter, sample_sharded=sharded)
    barrier(world)
    clocks = ClockSampler(local if world > 1 else 0, out_dir(args) / f"clocks_sharded_rank{rank}.csv")
    dev, launches, nodes = [], 0, 0
    split = {"eval_ms": 0.0, "comm_ms": 0.0, "step_ms": 0.0}
    st_sum = dict.fromkeys(("eval_ms", "flops", "node_evals", "sample_evals", "eval_launches"), 0)
    for _ in range(args.steps):
        co.fit_loaded(max_iter=max_iter, sample_sharded=sharded)
        st = co.stats()
        dev.append(st["device_ms"])
        launches += st["kernel_launches"]
        nodes += st["node_evals"]
        for k in split:
            split[k] += st[k] / args.steps
        for k in st_sum:
            st_sum[k] += st[k]
        passes = int(st["iters_run"]) + 1
    clk = clocks.stop()
    barrier(world)
    total_ms = max_over_ranks(float(sum(dev)), world)
    nodes_all = sum_over_ranks(float(nodes), world)
    # per-fit device time split of the slowest rank's figures (comm: chunk sum + all-reduce,
    # waiting for the other ranks included)
    split = {k: max_over_ranks(v, world) for k, v in split.items()}
    if rank != 0:
        return
    M = int(pop["M"])
    print(json.dumps({
        "metric": f"LM fits/sec (sample-sharded: M={M}, N={pop['N']}, {max_iter} iters, "
                  f"{precision})",
        "value": M * args.steps / (total_ms / 1e3), "unit": "fits/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32" if precision == "fp32" else "f64", "data": "synthetic",
        "config": {"workload": "sharded", "trees": M, "N": int(pop["N"]),
                   "max_iter": max_iter, "parallelism": f"sample-sharded x{world} "
                   "(NCCL all-reduce of JtJ/Jtr/loss per iteration)"},
        "node_evals_per_s": nodes_all / (total_ms / 1e3), "gpu_launches": launches,
        "per_fit_ms": {**split, "passes": passes},
        "roofline": {**config_roofline(st_sum, mine, precision, peaks), "rank": 0},
        "clocks": clk}),
        flush=True)


def run_profile_case(args) -> None:
    """Small case of the same kernel for ncu captures: --profile-trees trees (default 8,192)
    of the metric configuration, or of --config NAME (same N, same tree distribution), a few
    LM iterations."""
    from cusr_b200 import InProcessCO, synth

    pop = synth.make_config(args.config or CONFIG, M=args.profile_trees, seed=0)
    metas = np.asarray(pop["metas"])
    K = metas[:, 3]
    bins = {}
    for kc, lo, hi in ((4, 0, 4), (8, 5, 8), (12, 9, 12), (16, 13, 16), (32, 17, 32)):
        sel = (K >= lo) & (K <= hi)
        bins[str(kc)] = {"trees": int(sel.sum()), "nodes": int(metas[sel, 1].sum()),
                         "tree_samples": int(sel.sum()) * int(pop["N"])}
    print(json.dumps({"profile_bins": bins}), flush=True)
    co = InProcessCO(device_id=0, lib_path=args.profile_lib)
    precision = args.profile_precision or pop["precision"]
    co.load(pop, precision=precision)
    kw = {}
    if args.profile_alg == "trust_region":
        kw = dict(algorithm="trust_region", xtol=1e-10, tr_dd=args.profile_tr_dd)
    res = co.fit_loaded(max_iter=args.profile_iters, **kw)
    st = co.stats()
    print(json.dumps({"profile_case": True, "lib": args.profile_lib or "in-tree",
                      "trees": int(pop["M"]), "N": int(pop["N"]),
                      "iters": args.profile_iters, "device_ms": st["device_ms"],
                      "eval_launches": st["eval_launches"], "flops": st["flops"],
                      "eval_ms": st["eval_ms"], "node_evals": st["node_evals"],
                      "statuses": np.bincount(res["status"], minlength=5).tolist()}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference_gpu"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity-mode", action="store_true",
                    help="skip the parity-grade mode's measurement")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's CUDA path (--impl reference and the default arm)")
    ap.add_argument("--out-dir", default=None,
                    help="directory for report files (default $CUSR_REPORT_DIR, else a temp dir)")
    ap.add_argument("--profile-case", action="store_true",
                    help="run the small ncu case (--profile-trees trees) instead of the benchmark")
    ap.add_argument("--profile-iters", type=int, default=2)
    ap.add_argument("--profile-trees", type=int, default=8192)
    ap.add_argument("--profile-alg", choices=["reference", "trust_region"], default="reference",
                    help="--profile-case: the LM algorithm of the fit")
    ap.add_argument("--profile-tr-dd", action="store_true",
                    help="--profile-case with --profile-alg trust_region: double-double normal "
                         "equations (CoOptions.tr_dd; fp64)")
    ap.add_argument("--profile-lib", default=None,
                    help="--profile-case: a variant build of the library (python -m "
                         "cusr_b200.build --define ... --lib PATH)")
    ap.add_argument("--profile-precision", default=None,
                    help="--profile-case: fp32 | fp64 | fp32_fast (default: the config's)")
    ap.add_argument("--config", default=None,
                    help="bench one BASELINE configuration instead of the headline metric: "
                         "pr1, mid, physics, long, scale, sharded")
    ap.add_argument("--fast-math", action="store_true",
                    help="--config: run fp32 configurations with CO_PREC_FP32_FAST")
    ap.add_argument("--sample-sharded", action="store_true",
                    help="the sample-sharded configuration (M=512, N=10M) over all ranks")
    ap.add_argument("--M", type=int, default=None)
    ap.add_argument("--N", type=int, default=None)
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
        return
    world, rank, local = dist_setup()
    try:
        if args.config:
            run_config(args, world, rank, local)
        elif args.sample_sharded:
            run_sample_sharded(args, world, rank, local)
        elif args.impl == "reference":
            run_reference(args, world, rank)
        elif args.impl == "reference_gpu":
            run_reference_gpu(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
