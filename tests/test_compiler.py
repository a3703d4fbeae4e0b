"""Host-side tests of the bytecode compiler (pop.bin prefix trees -> register-stack
programs): the compiled program, run by the library's host emulation, reproduces the oracle's
value and reverse-mode gradient; malformed trees are rejected."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _helpers import conditioned_close, fixture_pop, make_tree, pop1000
from cusr_b200 import co_inproc, popio, synth
from oracle import interp

LIB = ctypes.CDLL(str(co_inproc.default_lib_path()))
LIB.cusr_eval_program.restype = ctypes.c_double
VP = ctypes.c_void_p


def compile_tree(nt, nv, ci, K, n_vars):
    nt = np.ascontiguousarray(nt, np.int32)
    nv = np.ascontiguousarray(nv, np.float32)
    ci = np.ascontiguousarray(ci, np.int32)
    code = np.zeros(2048, np.uint32)
    info = np.zeros(5, np.int32)
    rc = LIB.cusr_compile_tree(nt.ctypes.data_as(VP), nv.ctypes.data_as(VP), ci.ctypes.data_as(VP),
                               len(nt), int(K), int(n_vars), code.ctypes.data_as(VP), 2048,
                               info.ctypes.data_as(VP))
    nf, nb = int(info[0]), int(info[4])
    fwd, bwd = code[:nf].copy(), code[nf:nf + nb].copy()
    table = code[nf + nb:nf + nb + (int(K) + 4) // 4].copy()
    return rc, (fwd, bwd, table), info


def row_slots(table, K):
    """Tape slot of each gradient row (K entries) and of the residual row."""
    b = np.asarray(table, np.uint32).view(np.uint8)
    return [int(s) for s in b[:K + 1]]


def run_program(code, x, c, K):
    fwd, bwd, table = code
    rev = np.ascontiguousarray(np.concatenate([bwd, table]), np.uint32)
    x = np.ascontiguousarray(x, np.float64)
    c = np.ascontiguousarray(c if len(c) else [0.0], np.float64)
    g = np.zeros(max(K, 1))
    v = LIB.cusr_eval_program(fwd.ctypes.data_as(VP), len(fwd), rev.ctypes.data_as(VP), len(bwd),
                              x.ctypes.data_as(VP), c.ctypes.data_as(VP), int(K),
                              g.ctypes.data_as(VP))
    return v, g[:K]


def check_pop(pop, max_samples=24):
    n_checked = 0
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        rc, code, info = compile_tree(nt, nv, ci, K, pop["n_vars"])
        assert rc == 0
        # Sethi-Ullman order never needs more spill slots than the reference stack depth
        assert info[1] <= max(popio.stack_depth(nt) - 1, 0)
        off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][off:off + K], np.float64)
        xs = np.asarray(pop["xs"][:max_samples], np.float64)
        y, J = interp.value_and_jacobian(nt, nv, ci, xs, c)
        S = interp.error_scale(nt, nv, ci, xs, c)
        for i in range(xs.shape[0]):
            v, g = run_program(code, xs[i], c, K)
            assert conditioned_close(v, y[i], S[i], 1e-12, 2.0 ** -53).all(), (m, i, v, y[i])
            well = np.isfinite(y[i]) and S[i] < 1e6 * max(abs(y[i]), 1e-300)
            if K and well:
                ok = np.isfinite(J[i])
                assert np.allclose(g[ok], J[i][ok], rtol=1e-9, atol=1e-9 * max(1.0, np.max(np.abs(J[i][ok]), initial=0))), (m, i)
            n_checked += 1
    return n_checked


def test_compiled_pr1_trees_match_oracle():
    assert check_pop(synth.make_config("pr1", M=96, N=32, seed=11)) > 0


def test_compiled_long_trees_match_oracle():
    assert check_pop(synth.make_config("long", M=12, N=8, seed=2), max_samples=8) > 0


def test_compiled_reference_fixtures_match_oracle():
    for name in ("pop_fixture", "pop_fixture_op", "pop_fixture_stress", "pop_fixture_scale_1e0"):
        check_pop(fixture_pop(name), max_samples=16)


def test_compiled_pop1000_match_oracle():
    pop, _ = pop1000()
    check_pop(popio.slice_pop(pop, 120), max_samples=8)


@pytest.mark.parametrize("fid", [14, 15, 16, 17, 18, 19, 20, 21, 22, 23, 24, 25, 26, 27, 28, 99])
def test_every_unary_operator(fid):
    nt, nv, ci = make_tree([("b", 3), ("c",), ("u", fid), ("b", 1), ("v", 0), ("c",)])
    rc, code, _ = compile_tree(nt, nv, ci, 2, 1)
    assert rc == 0
    xs = np.array([[0.3], [1.7], [-0.4]])
    c = np.array([0.8, 0.25])
    y, J = interp.value_and_jacobian(nt, nv, ci, xs, c)
    for i in range(3):
        v, g = run_program(code, xs[i], c, 2)
        np.testing.assert_allclose(v, y[i], rtol=1e-13, equal_nan=True)
        np.testing.assert_allclose(g, J[i], rtol=1e-12, atol=1e-300, equal_nan=True)


@pytest.mark.parametrize("fid", [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 99])
@pytest.mark.parametrize("shape", ["leaf_right", "leaf_left", "both_subtrees", "const_right"])
def test_every_binary_operator(fid, shape):
    sub_l = [("b", 3), ("c",), ("v", 0)]               # c0 * x0
    sub_r = [("u", 22), ("b", 2), ("v", 1), ("c",)]     # exp(x1 - c)
    if shape == "leaf_right":
        nodes = [("b", fid)] + sub_l + [("v", 1)]
    elif shape == "leaf_left":
        nodes = [("b", fid), ("v", 1)] + sub_l
    elif shape == "const_right":
        nodes = [("b", fid)] + sub_l + [("c",)]
    else:
        nodes = [("b", fid)] + sub_l + sub_r
    nt, nv, ci = make_tree(nodes)
    K = int((nt == 1).sum())
    rc, code, _ = compile_tree(nt, nv, ci, K, 2)
    assert rc == 0
    xs = np.array([[0.7, 1.3], [1.9, 0.2], [0.5, 0.5]])
    c = np.array([1.3, 0.6, 0.9])[:K]
    y, J = interp.value_and_jacobian(nt, nv, ci, xs, c)
    for i in range(3):
        v, g = run_program(code, xs[i], c, K)
        np.testing.assert_allclose(v, y[i], rtol=1e-13, equal_nan=True)
        np.testing.assert_allclose(g, J[i], rtol=1e-12, atol=1e-300, equal_nan=True)


def test_deep_spill_stack():
    # full binary tree of depth 6 with subtree operands at every level: spills needed
    def full(d):
        if d == 0:
            return [("b", 3), ("c",), ("v", 0)]
        return [("b", 1 if d % 2 else 4)] + full(d - 1) + full(d - 1)
    nt, nv, ci = make_tree(full(6))
    K = int((nt == 1).sum())
    rc, code, info = compile_tree(nt, nv, ci, K, 1)
    assert rc == 0 and info[1] >= 4
    xs = np.array([[1.1], [0.4]])
    c = np.linspace(0.5, 1.5, K)
    y, J = interp.value_and_jacobian(nt, nv, ci, xs, c)
    for i in range(2):
        v, g = run_program(code, xs[i], c, K)
        np.testing.assert_allclose(v, y[i], rtol=1e-12)
        np.testing.assert_allclose(g, J[i], rtol=1e-10, atol=1e-12)


def test_reverse_program_drops_no_op_instructions():
    # c0 * x0 + x1: the "+ x1" has no reverse work
    nt, nv, ci = make_tree([("b", 1), ("b", 3), ("c",), ("v", 0), ("v", 1)])
    rc, (fwd, bwd, table), info = compile_tree(nt, nv, ci, 1, 2)
    assert rc == 0 and len(bwd) < len(fwd)
    v, g = run_program((fwd, bwd, table), np.array([2.0, 3.0]), np.array([0.5]), 1)
    assert v == pytest.approx(4.0) and g[0] == pytest.approx(2.0)


def test_repeated_constant_rank_accumulates():
    # c0 * x0 + c0 (rank 0 twice): gradient x0 + 1, program marks constants non-unique
    nt, nv, ci = make_tree([("b", 1), ("b", 3), ("c",), ("v", 0), ("c",)])
    ci = np.array([-1, -1, 0, -1, 0], np.int32)
    rc, code, info = compile_tree(nt, nv, ci, 1, 1)
    assert rc == 0 and info[3] == 0
    v, g = run_program(code, np.array([2.5]), np.array([0.5]), 1)
    assert v == pytest.approx(0.5 * 2.5 + 0.5) and g[0] == pytest.approx(3.5)


@pytest.mark.parametrize("bad", ["underflow", "two_roots", "bad_type", "var_range", "ci_range"])
def test_malformed_trees_rejected(bad):
    nt, nv, ci = make_tree([("b", 1), ("v", 0), ("c",)])
    K, n_vars = 1, 1
    if bad == "underflow":
        nt, nv, ci = nt[:2], nv[:2], ci[:2]
    elif bad == "two_roots":
        nt, nv, ci = make_tree([("v", 0), ("c",)])
    elif bad == "bad_type":
        nt = nt.copy(); nt[1] = 4
    elif bad == "var_range":
        nv = nv.copy(); nv[1] = 3.0
    else:
        ci = ci.copy(); ci[2] = 5
    rc, _, _ = compile_tree(nt, nv, ci, K, n_vars)
    assert rc == co_inproc.CO_ERR_BADTREE


def test_program_limits():
    # 1024 nodes exceed the per-tree node limit
    nodes = [("u", 25)] * 1023 + [("v", 0)]
    nt, nv, ci = make_tree(nodes)
    rc, _, _ = compile_tree(nt, nv, ci, 0, 1)
    assert rc == co_inproc.CO_ERR_BOUNDS


# reverse opcodes (cusr_b200/csrc/program.h, enum BOp) and the row-write flag
(B_GRAD, B_GRAD_RESTORE, B_RESTORE, B_GRAD_NEG, B_SPILL, B_SPILL_NEG, B_NEG, B_GRAD_THEN_NEG,
 B_SPILL_THEN_NEG, B_SCALE_X, B_SCALE_T0, B_MULC, B_GRAD_T1_T0, B_SPILL_T1_T0, B_GRAD_1MT0_T0,
 B_SPILL_1MT0_T0, B_ZERO, B_GRAD_ZERO, B_SPILL_ZERO, B_SCALE_1MT0, B_SCALE2_T, B_ROW_ZERO) = range(22)
B_ACC = 32
ROW_WRITES = {B_GRAD, B_GRAD_RESTORE, B_GRAD_NEG, B_GRAD_THEN_NEG, B_MULC, B_GRAD_T1_T0,
              B_GRAD_1MT0_T0, B_GRAD_ZERO}


def tape_reads(w):
    op, idx, ts = w & 31, (w >> 8) & 255, w >> 24
    if op in (B_SCALE_T0, B_MULC, B_GRAD_1MT0_T0, B_SPILL_1MT0_T0, B_SCALE_1MT0):
        return [ts]
    if op in (B_GRAD_T1_T0, B_SPILL_T1_T0):
        return [ts, ts + 1]
    if op == B_SCALE2_T:
        return [ts, idx]
    return []


def row_of(w):
    """Row slot named by a row-writing word (ts for B_GRAD_RESTORE, else sd)."""
    return (w >> 24) if (w & 31) == B_GRAD_RESTORE else ((w >> 16) & 255)


def forward_tape_slots(fwd):
    """Slots the forward program writes (one past the highest)."""
    hi = 0
    for w in fwd:
        code, ts = int(w) & 255, int(w) >> 24
        if code >= 8:   # operators; two-slot partials may use ts + 1
            hi = max(hi, ts + 2)
    return hi


@pytest.mark.parametrize("name", ["metric", "long"])
def test_gradient_rows_live_in_dead_tape_slots(name):
    pop = synth.make_config(name, M=300, N=16, seed=3)
    extra = []
    for m in range(pop["M"]):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        if K == 0:
            continue
        rc, (fwd, bwd, table), info = compile_tree(nt, nv, ci, K, pop["n_vars"])
        assert rc == 0
        slots = row_slots(table, K)
        n_slots = int(info[2])
        assert all(s < n_slots for s in slots)
        bwd = [int(w) for w in bwd]
        present = sorted({int(k) for k in ci[nt == 1]})
        # distinct rows for distinct constants, one shared zero row for absent ones, the
        # residual row apart from all of them
        grad_slots = {slots[k] for k in present}
        assert len(grad_slots) == len(present)
        assert slots[K] not in grad_slots
        absent = [k for k in range(K) if k not in present]
        if absent:
            zero = {slots[k] for k in absent}
            assert len(zero) == 1 and not (zero & grad_slots) and slots[K] not in zero
            assert bwd[-1] & 31 == B_ROW_ZERO and bwd[-1] >> 24 == slots[absent[0]]
        # the first write of each row stores, later ones add; a row's slot is never read as
        # tape after its first write
        first = {}
        for p, w in enumerate(bwd):
            op = w & 31
            if op in ROW_WRITES:
                s = row_of(w)
                assert s in grad_slots and s == slots[(w >> 8) & 255]
                if s not in first:
                    first[s] = p
                    assert not (w & B_ACC)
                else:
                    assert w & B_ACC
            else:
                assert not (w & B_ACC)
        for p, w in enumerate(bwd):
            for s in tape_reads(w):
                assert s not in first or p <= first[s], (m, p, s)
        extra.append(n_slots - forward_tape_slots(fwd))
    # rows almost always fit in slots the reverse sweep has finished with
    assert np.mean(extra) < 1.0


def test_absent_constant_gets_the_zero_row():
    # c0 * x0 + c2 with K = 3 (rank 1 unused): its gradient is exactly 0
    nt, nv, ci = make_tree([("b", 1), ("b", 3), ("c",), ("v", 0), ("c",)])
    ci = np.array([-1, -1, 0, -1, 2], np.int32)
    rc, code, info = compile_tree(nt, nv, ci, 3, 1)
    assert rc == 0
    fwd, bwd, table = code
    assert int(bwd[-1]) & 31 == B_ROW_ZERO
    v, g = run_program(code, np.array([1.5]), np.array([2.0, 7.0, -1.0]), 3)
    assert v == pytest.approx(2.0 * 1.5 - 1.0)
    np.testing.assert_array_equal(g, [1.5, 0.0, 1.0])
