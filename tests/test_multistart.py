"""Multi-start host side: the start-point generator's host restatement against the engine's
own formulas compiled for the host (cusr_start_points), determinism, start 0 = c_init, the
kinds' spread; and the parity preset's options reach the ABI. The device fits themselves are
in test_gpu_fit.py."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from cusr_b200 import co_inproc, multistart, synth


def _host_points(lib, pop, S, seed):
    out = []
    for m in range(int(pop["M"])):
        _o, _n, c_off, K = (int(v) for v in pop["metas"][m])
        c0 = np.ascontiguousarray(pop["c_init"][c_off:c_off + K], np.float32)
        buf = np.zeros(max(S * K, 1), np.float32)
        lib.cusr_start_points(ctypes.c_uint64(seed), ctypes.c_int64(m), S, K,
                              c0.ctypes.data_as(ctypes.c_void_p), buf.ctypes.data_as(ctypes.c_void_p))
        out.append(buf[:S * K])
    return np.concatenate(out)


@pytest.fixture(scope="module")
def lib():
    path = co_inproc.default_lib_path()
    if not path.exists():
        pytest.skip("library not built")
    lib = ctypes.CDLL(str(path))
    lib.cusr_start_points.restype = None
    return lib


def test_start_points_match_engine_formulas(lib):
    pop = synth.make_config("pr1", M=40, N=8, seed=3)
    for S, seed in ((1, 0), (9, 0), (20, 12345), (33, 2 ** 63 + 7)):
        mine = multistart.start_points(pop, S, seed)
        host = _host_points(lib, pop, S, seed)
        assert mine.shape == host.shape
        # the same formulas in numpy and C: equal floats, at most one float ulp apart where
        # the two libm's round log / cos / exp differently
        assert np.array_equal(mine, host) or np.max(
            np.abs(mine.view(np.int32).astype(np.int64) - host.view(np.int32))) <= 1


def test_start_points_first_is_c_init_and_deterministic():
    pop = synth.make_config("pr1", M=20, N=8, seed=3)
    a = multistart.start_points(pop, 8, seed=5)
    np.testing.assert_array_equal(a, multistart.start_points(pop, 8, seed=5))
    assert not np.array_equal(a, multistart.start_points(pop, 8, seed=6))
    K = pop["metas"][:, 3]
    off = 0
    for m in range(20):
        k = int(K[m])
        c0 = pop["c_init"][pop["metas"][m][2]:pop["metas"][m][2] + k]
        np.testing.assert_array_equal(a[off:off + k], c0)          # start 0
        off += 8 * k


def test_start_kinds_spread():
    """Fresh N(0,1) / N(0,9) starts have those spreads."""
    pop = synth.make_config("pr1", M=256, N=4, seed=1)
    S = 9
    pts = multistart.start_points(pop, S, seed=0).astype(np.float64)
    K = pop["metas"][:, 3]
    start = np.repeat(np.tile(np.arange(S), 256), np.repeat(K, S))
    fresh1 = pts[(start > 0) & ((start - 1) % 4 == 2)]
    fresh3 = pts[(start > 0) & ((start - 1) % 4 == 3)]
    assert abs(np.std(fresh1) - 1.0) < 0.1 and abs(np.mean(fresh1)) < 0.1
    assert abs(np.std(fresh3) - 3.0) < 0.3


def test_parity_preset_reaches_options():
    opt = co_inproc.CoOptions()
    co_inproc.start_options(opt, **{k: v for k, v in co_inproc.PARITY.items()
                                    if k in ("algorithm", "n_starts", "tr_starts", "wave1",
                                             "ftol", "gtol")})
    assert opt.algorithm == 1 and opt.n_starts == 128 and opt.tr_starts == 128 and opt.wave1 == 8
    assert opt.ftol == 1e-10 and opt.gtol == 1e-8
    with pytest.raises(ValueError):
        co_inproc.start_options(opt, algorithm="newton")


def test_preset_keywords():
    kw = multistart.preset_kwargs(co_inproc.PARITY)
    assert kw["starts"] == 128 and kw["tr_starts"] == 128 and "algorithm" not in kw
    assert kw["explore_precision"] == "fp32" and kw["precision"] == "fp64"
    assert kw["polish_starts"] == 8 and kw["explore_max_iter"] == 30
    assert multistart.preset_kwargs(co_inproc.PARITY_FAST)["polish_starts"] == 1
    assert multistart.preset_kwargs(co_inproc.PARITY_MAX)["dd_starts"] == 16
    fp64 = multistart.preset_kwargs(co_inproc.PARITY_FP64)
    assert fp64["starts"] == 96 and fp64["explore_precision"] is None
    # every preset key is a fit_multistart parameter
    import inspect
    params = inspect.signature(multistart.fit_multistart).parameters
    for p in (co_inproc.PARITY, co_inproc.PARITY_FAST, co_inproc.PARITY_FP64, co_inproc.PARITY_MAX):
        assert set(multistart.preset_kwargs(p)) <= set(params) | {"ftol", "gtol"}


def test_dd_stage_batches_by_memory(monkeypatch):
    """The double-double stage splits a population into batches of consecutive trees when its
    per-sample Jacobians would exceed DD_BATCH_BYTES, and returns the outputs in tree order."""
    pop = synth.make_config("pr1", M=10, N=64, seed=2)
    calls = []

    class FakeCo:
        def optimize_ex(self, p, **kw):
            assert kw["tr_dd"] and kw["precision"] == "fp64"
            M = int(p["M"])
            calls.append(M)
            K = np.asarray(p["metas"]).reshape(M, 4)[:, 3]
            # each tree's constants, status and loss name the tree by its first constant
            return {"c_final": np.asarray(p["c_init"], np.float64),
                    "status": np.zeros(M, np.int32),
                    "loss_final": np.asarray([p["c_init"][o] if k else 0.0 for o, k in
                                              zip(np.asarray(p["metas"])[:, 2], K)]),
                    "iters": np.full(M, 3, np.int32)}

    kmax = int(np.asarray(pop["metas"])[:, 3].max())
    per_tree = 4 * (kmax + 1) * 64 * 8
    monkeypatch.setattr(multistart, "DD_BATCH_BYTES", 3 * per_tree)
    out = multistart._dd_stage(FakeCo(), pop, 4, 50, 1e-10, 0, {})
    assert calls == [3, 3, 3, 1]
    np.testing.assert_array_equal(out["c_final"], np.asarray(pop["c_init"], np.float64))
    assert out["status"].shape == (10,)
