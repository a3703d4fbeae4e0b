"""The batch_lm-compatible command-line front end (cusr_b200/batch_lm_b200): argument and
file handling on CPU; a fit through it on the GPU, read back exactly as the reference's
subprocess callers read it (backends.CudaKernelPop: status.bin, c_final.bin and the
"总耗时 X 秒" line; kernel_bridge._run_kernel: --quiet --max-iter)."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from _helpers import fixture_pop
from cusr_b200 import popio, synth

CLI = Path(__file__).resolve().parent.parent / "cusr_b200" / "batch_lm_b200"
TIME_RE = re.compile(r"总耗时 ([\d.]+) 秒")   # the reference caller's regex


def _run(*args):
    if not CLI.exists():
        pytest.skip("batch_lm_b200 not built")
    return subprocess.run([str(CLI), *map(str, args)], capture_output=True, encoding="utf-8",
                          timeout=600)


def test_cli_usage_and_missing_file(tmp_path):
    r = _run()
    assert r.returncode == 1 and "usage" in r.stderr
    r = _run(tmp_path / "nope.bin")
    assert r.returncode == 1


def test_cli_rejects_bad_magic(tmp_path):
    p = tmp_path / "bad.bin"
    p.write_bytes(b"\0" * 64)
    assert _run(p, tmp_path).returncode == 1


def test_cli_bounds_exit_code(tmp_path):
    """K_max beyond 32 exits 2 before any device work, as the reference binary."""
    pop = synth.make_config("pr1", M=4, N=16, seed=0)
    pop = dict(pop)
    pop["K_max"] = 40
    p = tmp_path / "pop.bin"
    popio.save_pop_bin(pop, p)
    assert _run(p, tmp_path, "--quiet").returncode == 2


def test_cli_links_reference_names():
    if not CLI.exists():
        pytest.skip("batch_lm_b200 not built")
    for name in ("batch_lm", "batch_lm_ad"):
        assert (CLI.parent / name).resolve() == CLI.resolve()


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp32", "fp64"])
def test_cli_fit_matches_library(tmp_path, precision):
    from cusr_b200 import get_inproc_co

    pop = fixture_pop("pop_fixture_op")
    p = tmp_path / "pop.bin"
    popio.save_pop_bin(pop, p)
    r = _run(p, tmp_path, "--max-iter", 40, "--precision", precision)
    assert r.returncode == 0, r.stderr
    m = TIME_RE.search(r.stdout)
    assert m and float(m.group(1)) > 0
    status = np.fromfile(tmp_path / "status.bin", np.int32)
    c_final = np.fromfile(tmp_path / "c_final.bin", np.float32)
    lf = np.fromfile(tmp_path / "loss_final.bin", np.float32)
    co = get_inproc_co(0)
    if precision == "fp32":
        ref = co.optimize(pop, max_iter=40)
    else:
        ref = co.optimize_ex(pop, max_iter=40, precision="fp64")
    np.testing.assert_array_equal(status, ref["status"])
    np.testing.assert_array_equal(c_final, np.asarray(ref["c_final"]).astype(np.float32))
    np.testing.assert_array_equal(lf, np.asarray(ref["loss_final"]).astype(np.float32))
    # --quiet prints nothing and writes the same blobs
    q = _run(p, tmp_path / ".." / tmp_path.name, "--quiet", "--max-iter", 40,
             "--precision", precision)
    assert q.returncode == 0 and q.stdout == ""
    np.testing.assert_array_equal(np.fromfile(tmp_path / "c_final.bin", np.float32), c_final)


@pytest.mark.gpu
def test_parity_gate_through_cli(tmp_path):
    """The reference's kernel replacement gate (cusr/kernel/tests/test_parity_gate.py with
    verify.py's definitions) on its own pop.bin fixture, run through the command line as the
    gate runs the binary: loss-down rate (K>0) >= 93%, gpu_loss <= max(1.05x, +1e-10) of the
    scipy fit on trees both converged >= 90%, within 10x >= 99%."""
    from _helpers import pop1000
    from oracle import interp

    pop, g = pop1000()
    p = tmp_path / "pop.bin"
    popio.save_pop_bin(pop, p)
    r = _run(p, tmp_path)
    assert r.returncode == 0, r.stderr
    status = np.fromfile(tmp_path / "status.bin", np.int32)
    c_final = np.fromfile(tmp_path / "c_final.bin", np.float32).astype(np.float64)
    gpu_loss = interp.loss_pop(pop, c_final)
    gpu_init = interp.loss_pop(pop, pop["c_init"].astype(np.float64))
    sc_loss, sc_ok = g["scipy/loss64"], g["scipy/status"] == 0
    K = np.asarray(pop["metas"])[:, 3]
    elig = (K > 0) & np.isfinite(gpu_loss) & np.isfinite(gpu_init)
    loss_down = float(np.mean(gpu_loss[elig] < gpu_init[elig]))
    both = (K > 0) & sc_ok & (status == 0)
    fin = both & np.isfinite(gpu_loss) & np.isfinite(sc_loss)

    def env(k):
        return float(np.sum(gpu_loss[fin] <= np.maximum(k * sc_loss[fin], sc_loss[fin] + 1e-10))
                     / max(int(both.sum()), 1))

    rates = {"loss_down": loss_down, "within_1.05": env(1.05), "within_10": env(10.0),
             "both_converged": int(both.sum())}
    from _helpers import write_report

    write_report("parity_gate_pop1000.json", rates)
    assert rates["loss_down"] >= 0.93, rates
    assert rates["within_1.05"] >= 0.90, rates
    assert rates["within_10"] >= 0.99, rates
