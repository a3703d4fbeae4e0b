"""pop.bin I/O and the seeded synthetic configurations."""
from __future__ import annotations

import numpy as np
import pytest

from _helpers import fixture_pop
from cusr_b200 import popio, synth
from oracle import interp


def test_roundtrip_is_byte_identical(tmp_path):
    pop = fixture_pop("pop_fixture_op")
    p1 = tmp_path / "a.bin"
    popio.save_pop_bin(pop, p1)
    back = popio.load_pop_bin(p1)
    p2 = tmp_path / "b.bin"
    popio.save_pop_bin(back, p2)
    assert p1.read_bytes() == p2.read_bytes()
    assert len(p1.read_bytes()) == 64 + 12 * pop["total_nodes"] + 16 * pop["M"] + 4 * (
        pop["total_c"] + pop["N"] * pop["n_vars"] + pop["M"] * pop["N"])
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        np.testing.assert_array_equal(back[k], pop[k])


def test_bad_magic_rejected(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"\0" * 64)
    with pytest.raises(ValueError):
        popio.load_pop_bin(p)


def test_build_pop_invariants():
    pop = synth.make_config("pr1", M=40, N=50, seed=3)
    assert pop["metas"][:, 1].sum() == pop["total_nodes"]
    assert pop["metas"][:, 3].sum() == pop["total_c"]
    assert pop["K_max"] == pop["metas"][:, 3].max()
    assert pop["max_stack"] == max(popio.stack_depth(interp.tree_view(pop, m)[0])
                                   for m in range(40))
    with pytest.raises(ValueError):
        popio.build_pop([(np.array([1], np.int32), np.zeros(1, np.float32),
                          np.array([3], np.int32), [1.0])], pop["xs"], pop["ym"][None])


def test_slice_and_replicate():
    pop = synth.make_config("pr1", M=30, N=20, seed=4)
    sub = popio.slice_pop(pop, [3, 7, 11])
    assert sub["M"] == 3
    for j, m in enumerate([3, 7, 11]):
        a = interp.tree_view(pop, m)
        b = interp.tree_view(sub, j)
        np.testing.assert_array_equal(a[0], b[0])
    rep = popio.replicate_ym(sub)
    assert rep["ym"].shape == (3, 20) and np.all(rep["ym"] == pop["ym"])


@pytest.mark.parametrize("name", ["pr1", "mid", "long", "physics"])
def test_configs_are_seeded_and_in_range(name):
    a = synth.make_config(name, M=24, N=64, seed=9)
    b = synth.make_config(name, M=24, N=64, seed=9)
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        np.testing.assert_array_equal(a[k], b[k])
    cfg = synth.CONFIGS[name]
    K = a["metas"][:, 3]
    assert K.min() >= cfg["K"][0] and K.max() <= cfg["K"][1]
    if "len" in cfg:
        n = a["metas"][:, 1]
        assert n.min() >= cfg["len"][0] and n.max() <= cfg["len"][1]
    # every tree is finite at its initial constants on the check subset
    for m in range(24):
        nt, nv, ci, _y, Km = interp.tree_view(a, m)
        off = int(a["metas"][m][2])
        y = interp.eval_tree_arrays(nt, nv, ci, a["xs"][:64], a["c_init"][off:off + Km])
        assert np.all(np.isfinite(y))


@pytest.mark.parametrize("fixture,name", [("configs_full_scipy.npz", "mid"),
                                          ("configs_full_scipy.npz", "physics"),
                                          ("configs_full_scipy.npz", "long"),
                                          ("configs_full_scipy.npz", "scale"),
                                          ("sharded_scipy.npz", "sharded")])
def test_full_n_fixtures_regenerate_from_the_seeded_generator(fixture, name):
    """The full-N scipy fixtures store their inputs as a digest; the GPU parity tests
    regenerate them with the seeded generator. Same bytes here, on the CPU."""
    import hashlib

    from _helpers import GOLDEN

    z = np.load(GOLDEN / fixture)
    pop = synth.make_config(name, M=int(z[f"{name}/M"]), seed=11)
    h = hashlib.sha256()
    for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym"):
        h.update(np.ascontiguousarray(pop[k]).tobytes())
    assert h.hexdigest() == str(z[f"{name}/digest"])
    for k in ("nt", "ci", "metas", "c_init"):
        np.testing.assert_array_equal(np.asarray(pop[k]), z[f"{name}/{k}"])
