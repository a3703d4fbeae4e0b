"""In-loop amortisation (the reference's test_inproc_amortize.py semantics) and resident
inputs across calls (CoOptions.keep_inputs):
  * one CUDA context for the handle's lifetime (driver-API handle stable across calls);
  * repeated fits of one population take index-independent time (no per-call re-init);
  * the setup / loop split is reported and the loop dominates a real population;
  * keep_inputs: a new population on the X / shared y already on the device gives exactly
    the result of a call that uploads them, warm starts from a parent's constants work, and
    an incompatible resident state is refused with CO_ERR_NULLARG.
"""
from __future__ import annotations

import ctypes
import statistics
import time

import numpy as np
import pytest

from cusr_b200 import InProcessCO, popio, synth
from cusr_b200.co_inproc import CO_ERR_NULLARG, COError
from oracle import interp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def co():
    c = InProcessCO(device_id=0)
    yield c
    c.teardown()


def _current_ctx() -> int:
    cuda = ctypes.CDLL("libcuda.so.1")
    h = ctypes.c_void_p()
    assert cuda.cuCtxGetCurrent(ctypes.byref(h)) == 0
    return int(h.value or 0)


def _trees(pop):
    out = []
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        off = int(pop["metas"][m][2])
        out.append((nt, nv, ci, pop["c_init"][off:off + K]))
    return out


def test_primary_context_created_once(co):
    pop = synth.make_config("mid", M=256, N=2000, seed=1)
    co.optimize(pop, max_iter=5)
    h0 = _current_ctx()
    assert h0 != 0
    for _ in range(3):
        co.optimize(pop, max_iter=5)
        assert _current_ctx() == h0


def test_co_optimize_wall_index_independent(co):
    pop = synth.make_config("mid", M=2048, N=4000, seed=2)
    co.optimize(pop, max_iter=20)            # warm-up: lazy module load
    walls = []
    for _ in range(8):
        t0 = time.perf_counter()
        co.optimize(pop, max_iter=20)
        walls.append(time.perf_counter() - t0)
    med = statistics.median(walls)
    assert max(walls) <= 1.5 * med, walls
    assert statistics.mean(walls[4:]) <= 1.2 * statistics.mean(walls[:4]), walls


def test_setup_loop_split(co):
    """Once the context has seen the sizes (buffers grown, kernels loaded), the per-call
    setup (compile, upload, initial pass) is small against the LM loop."""
    pop = synth.make_config("mid", M=4096, N=10000, seed=3)
    co.optimize(pop, max_iter=50)        # first call: allocations and lazy kernel loading
    co.optimize(pop, max_iter=50)
    setup_ms, loop_ms = co.last_split()
    assert setup_ms > 0 and loop_ms > 0
    assert setup_ms < loop_ms


def test_keep_inputs_equals_full_upload(co):
    base = synth.make_config("mid", M=300, N=3000, seed=4)
    other = synth.make_config("mid", M=200, N=3000, seed=5)
    child = popio.build_pop(_trees(other), base["xs"], base["ym"])    # new trees, same data
    co.optimize_ex(base, max_iter=10)                                 # uploads X / y
    lean = {k: v for k, v in child.items() if k not in ("xs", "ym")}
    kept = co.optimize_ex(lean, max_iter=30, keep_inputs=True)
    full = co.optimize_ex(child, max_iter=30)
    for k in kept:
        assert kept[k].tobytes() == full[k].tobytes(), k
    # warm start from the parent's constants on the resident data (fp32 c_init)
    warm = dict(lean)
    warm["c_init"] = full["c_final"].astype(np.float32)
    again = co.optimize_ex(warm, max_iter=30, keep_inputs=True)
    fin = np.isfinite(full["loss_final"]) & (full["status"] != 3)
    assert np.all(again["loss_final"][fin] <= full["loss_final"][fin] * (1 + 1e-4) + 1e-9)


def test_keep_inputs_refused_without_compatible_state():
    fresh = InProcessCO(device_id=0)
    try:
        pop = synth.make_config("mid", M=50, N=500, seed=6)
        lean = {k: v for k, v in pop.items() if k not in ("xs", "ym")}
        with pytest.raises(COError) as e:
            fresh.optimize_ex(lean, keep_inputs=True)
        assert e.value.code == CO_ERR_NULLARG
        fresh.optimize_ex(pop, max_iter=5)
        other_n = synth.make_config("mid", M=50, N=700, seed=6)
        lean_n = {k: v for k, v in other_n.items() if k not in ("xs", "ym")}
        with pytest.raises(COError):
            fresh.optimize_ex(lean_n, keep_inputs=True)          # different N
        phys = synth.make_config("physics", M=20, N=500, seed=7)  # per-tree targets
        fresh.optimize_ex(phys, max_iter=5, precision="fp64")
        lean_p = {k: v for k, v in phys.items() if k not in ("xs", "ym")}
        with pytest.raises(COError):
            fresh.optimize_ex(lean_p, keep_inputs=True, precision="fp64")
    finally:
        fresh.teardown()
