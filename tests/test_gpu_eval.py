"""Device interpreter parity (the fused pass, through the C ABI co_evaluate): values,
reverse-mode Jacobians and normal-equation blocks against the CPU oracle, the reference's
interpreter vectors and its reverse-AD Jacobian samples.

Tolerances (written per test): fp64 1e-12 relative, fp32 1e-5 relative, each widened by
64 * unit roundoff * S where S = sum |df/dv_n| |v_n| over the tree's operator nodes (the
first-order rounding-error scale; it only matters for ill-conditioned samples such as
cos(exp(34)), where 1-ulp differences in library transcendentals are amplified)."""
from __future__ import annotations

import numpy as np
import pytest

from _helpers import GOLDEN, conditioned_close, load_npz_pop, make_tree, pop1000
from cusr_b200 import InProcessCO, popio, synth
from oracle import interp

pytestmark = pytest.mark.gpu

U64, U32 = 2.0 ** -53, 2.0 ** -24


@pytest.fixture(scope="module")
def co():
    c = InProcessCO(device_id=0)
    yield c
    c.teardown()


def _check_values(co, pop, precision, rel, unit, min_strict=0.97, fast_k=0.0):
    out = co.evaluate(pop, precision=precision, values=True)
    vals = out["values"]
    strict = total = 0
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][off:off + K], np.float64)
        if precision in ("fp32", "fp32_fast"):
            c = c.astype(np.float32).astype(np.float64)
        y = interp.eval_tree_arrays(nt, nv, ci, pop["xs"], c)
        S = interp.error_scale(nt, nv, ci, pop["xs"], c)
        hi, lo = interp.intermediate_range(nt, nv, ci, pop["xs"], c)
        if precision in ("fp32", "fp32_fast"):
            outside = (hi > 1e37) | (lo < 1e-30)   # not representable in normal fp32
        else:
            outside = np.zeros(y.shape, bool)
        if fast_k:
            S = S + fast_k / (64.0 * unit) * interp.FAST_MATH_UNIT * interp.fast_math_error_scale(
                nt, nv, ci, pop["xs"], c)
        ok = conditioned_close(vals[m], y, S, rel, unit) | outside
        assert ok.all(), (m, np.flatnonzero(~ok)[:5], vals[m][~ok][:5], y[~ok][:5])
        fin = np.isfinite(y) & ~outside
        with np.errstate(all="ignore"):
            strict += int(np.sum(np.abs(vals[m][fin] - y[fin]) <= rel * np.abs(y[fin]) + 1e-300))
        total += int(fin.sum())
    # the plain relative bound holds on nearly every sample (the rest are ill-conditioned)
    assert strict / max(total, 1) >= min_strict


def test_values_fp64_match_oracle(co):
    _check_values(co, synth.make_config("pr1", M=96, N=300, seed=0), "fp64", 1e-12, U64)


def test_values_fp32_match_oracle(co):
    _check_values(co, synth.make_config("pr1", M=96, N=300, seed=0), "fp32", 1e-5, U32)


def test_values_fp32_fast_match_oracle(co):
    """The reference kernel's numerics (--use_fast_math): hardware sin/cos/exp/log
    approximations (absolute error about 2^-21.4 on the primary range, growing with |x|),
    approximate division and square root, denormals flushed. Checked against the fp64 oracle
    with the fp32 condition-scaled bound plus 8x the intrinsics' published error bounds
    propagated through the tree (oracle fast_math_error_scale); most samples still meet a
    plain 1e-4 relative bound."""
    for pop in (synth.make_config("pr1", M=96, N=300, seed=0),
                synth.make_config("mid", M=64, N=700, seed=4)):
        _check_values(co, pop, "fp32_fast", 1e-5, U32, min_strict=0.85, fast_k=8.0)
        _report_fast_values(co, pop)


def _report_fast_values(co, pop):
    """Error statistics of the fast-math values against the fp64 oracle and the IEEE fp32
    path (written next to the GPU run's other parity reports)."""
    from _helpers import report_dir, write_report

    if report_dir() is None:
        return
    fast = co.evaluate(pop, precision="fp32_fast", values=True)["values"]
    ieee = co.evaluate(pop, precision="fp32", values=True)["values"]
    rel_f, rel_i = [], []
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][off:off + K], np.float32).astype(np.float64)
        y = interp.eval_tree_arrays(nt, nv, ci, pop["xs"], c)
        fin = np.isfinite(y) & (np.abs(y) > 1e-30)
        with np.errstate(all="ignore"):
            rel_f.append(np.abs(fast[m][fin] - y[fin]) / np.abs(y[fin]))
            rel_i.append(np.abs(ieee[m][fin] - y[fin]) / np.abs(y[fin]))
    rf, ri = np.concatenate(rel_f), np.concatenate(rel_i)
    q = [0.5, 0.9, 0.99, 0.999]
    write_report(f"fast_values_M{pop['M']}_N{pop['N']}.json",
                 {"fast_rel_quantiles": np.nanquantile(rf, q).tolist(),
                  "ieee_rel_quantiles": np.nanquantile(ri, q).tolist(),
                  "fast_within_1e-5": float(np.mean(rf <= 1e-5)),
                  "ieee_within_1e-5": float(np.mean(ri <= 1e-5))})


def test_values_mid_config_both_precisions(co):
    pop = synth.make_config("mid", M=64, N=700, seed=4)
    _check_values(co, pop, "fp64", 1e-12, U64)
    _check_values(co, pop, "fp32", 1e-5, U32, min_strict=0.9)


def test_values_match_reference_interp_vectors(co):
    z = np.load(GOLDEN / "interp_vectors.npz")
    pop = load_npz_pop(z, "pr1")
    vals = co.evaluate(pop, precision="fp64", values=True)["values"]
    for m in range(pop["M"]):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        off = int(pop["metas"][m][2])
        S = interp.error_scale(nt, nv, ci, pop["xs"], pop["c_init"][off:off + K])
        assert conditioned_close(vals[m], z["pr1/values"][m], S, 1e-12, U64).all(), m


def _check_jacobian(co, pop, precision, tol):
    out = co.evaluate(pop, precision=precision, values=False, jacobian=True)
    J_dev = out["jacobian"]
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        if K == 0:
            continue
        off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][off:off + K], np.float64)
        if precision in ("fp32", "fp32_fast"):
            c = c.astype(np.float32).astype(np.float64)
        y, J = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c)
        S = interp.error_scale(nt, nv, ci, pop["xs"], c)
        well = np.isfinite(y) & (S <= 1e2 * np.maximum(np.abs(y), 1e-3)) & np.all(np.isfinite(J), 1)
        if precision == "fp32":
            hi, lo = interp.intermediate_range(nt, nv, ci, pop["xs"], c)
            well &= (hi < 1e15) & (lo > 1e-15)
            # elements whose gradient an fp32 evaluation of the same rules (numpy) reproduces
            # to 1e-4: elsewhere fp32 itself cannot resolve the gradient (e.g. sin(exp(.)))
            _, J32 = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c.astype(np.float32),
                                               dtype=np.float32)
            J32 = J32.astype(np.float64)
            with np.errstate(all="ignore"):
                resolved = np.abs(J32 - J) <= 1e-4 * np.abs(J) + 1e-30
        else:
            resolved = np.ones(J.shape, bool)
        Jd = J_dev[m, :K].T
        for k in range(K):
            sel = well & resolved[:, k]
            col = J[sel, k]
            if col.size == 0:
                continue
            scale = max(float(np.max(np.abs(col))), 1e-30)
            # normwise per column, and elementwise for the elements fp32 resolves
            err = float(np.max(np.abs(Jd[sel, k] - col)))
            assert err <= tol * scale, (m, k, err, scale)
            if precision == "fp32":
                assert np.all(np.abs(Jd[sel, k] - col) <= 1e-2 * np.abs(col) + tol * scale), (m, k)


def test_jacobian_fp64_matches_oracle(co):
    _check_jacobian(co, synth.make_config("pr1", M=64, N=256, seed=2), "fp64", 1e-10)


def test_jacobian_fp32_matches_oracle(co):
    # fp32 gradients of trees up to 31 nodes: normwise 1e-3 per column (the reference's own
    # host AD tests accept rel < 1e-3 against central differences)
    _check_jacobian(co, synth.make_config("pr1", M=64, N=256, seed=2), "fp32", 1e-3)


def test_jacobian_matches_reference_revad_samples(co):
    """The reference's own reverse-AD gradients (fp32, experiments/revad_v5 samples)."""
    z = np.load(GOLDEN / "jac_sample.npz")
    trees, ys = [], []
    n = int(z["n"])
    for i in range(n):
        trees.append((z[f"{i}/nt"], z[f"{i}/nv"], z[f"{i}/ci"], z[f"{i}/c"]))
    # each sample tree carries its own points: evaluate tree by tree
    for i in range(n):
        x = z[f"{i}/x"]
        pop = popio.build_pop([trees[i]], x, np.zeros((1, x.shape[0]), np.float32))
        J = co.evaluate(pop, precision="fp32", values=False, jacobian=True)["jacobian"][0]
        rev = z[f"{i}/rev"]
        K = rev.shape[1]
        Jd = J[:K].T
        ok = np.isfinite(rev)
        assert np.all(np.isfinite(Jd[ok])), i
        scale = np.maximum(np.abs(rev[ok]), 1.0)
        assert np.all(np.abs(Jd[ok] - rev[ok]) <= 2e-4 * scale), i


def _ref_blocks(pop, m, c):
    """Oracle block and a magnitude bound of each entry's rounding error: Gram entries by
    sum |J_i||J_j|, Jtr and the loss by sum |J| (|f| + |y|) (r = f - y cancels near a fit)."""
    nt, nv, ci, y, K = interp.tree_view(pop, m)
    f, J = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c)
    y = np.asarray(y, np.float64)
    r = f - y
    fy = np.abs(f) + np.abs(y)
    tri = np.concatenate([J[:, i] @ J[:, :i + 1] for i in range(K)]) if K else np.zeros(0)
    mag = np.concatenate([np.abs(J[:, i]) @ np.abs(J[:, :i + 1]) for i in range(K)]) if K else np.zeros(0)
    return (np.concatenate([tri, J.T @ r, [0.5 * r @ r]]),
            np.concatenate([mag, np.abs(J).T @ fy, [np.abs(r) @ fy]]))


def _check_blocks(co, pop, precision, tol, max_cond=None):
    blocks = co.evaluate(pop, precision=precision, values=False, blocks=True)["blocks"]
    n = 0
    for m in range(int(pop["M"])):
        off, K = int(pop["metas"][m][2]), int(pop["metas"][m][3])
        c = np.asarray(pop["c_init"][off:off + K], np.float64)
        if precision in ("fp32", "fp32_fast"):
            c = c.astype(np.float32).astype(np.float64)
        ref, mag = _ref_blocks(pop, m, c)
        if not np.all(np.isfinite(ref)):
            continue
        nt, nv, ci, _y, _ = interp.tree_view(pop, m)
        S = interp.error_scale(nt, nv, ci, pop["xs"], c)
        f = interp.eval_tree_arrays(nt, nv, ci, pop["xs"], c)
        cond = max_cond if max_cond is not None else (1e2 if precision == "fp32" else 1e5)
        if np.max(S) / (np.sqrt(np.mean(f * f)) + 1e-3) > cond:
            continue   # ill-conditioned tree: checked by the value tests
        if precision == "fp32":
            hi, lo = interp.intermediate_range(nt, nv, ci, pop["xs"], c)
            if np.max(hi) > 1e30 or np.min(lo) < 1e-30:
                continue   # not representable in fp32
        # entries whose oracle magnitude is exactly 0 (a column the fp64 oracle cancels to 0)
        # get a floor of tol * 1e-12 * the block's largest magnitude
        lim = tol * (mag + 1e-12 * float(np.max(mag))) + 1e-300
        bad = np.flatnonzero(~(np.abs(blocks[m] - ref) <= lim))
        assert bad.size == 0, (m, bad[:4], blocks[m][bad[:4]], ref[bad[:4]], mag[bad[:4]])
        n += 1
    assert n > 0


def test_blocks_fp64_match_oracle(co):
    _check_blocks(co, synth.make_config("pr1", M=64, N=1000, seed=6), "fp64", 1e-10)


def test_blocks_fp32_match_oracle(co):
    _check_blocks(co, synth.make_config("pr1", M=64, N=1000, seed=6), "fp32", 2e-4)


def _sum_of_terms_pop(M, K_lo, K_hi, N, seed):
    """Well-conditioned trees with many constants: c0 + sum_k c_k * g_k(x), g in
    {x_j, sin x_j, exp(-x_j^2)-like products}; K = 17..32 exercises the cooperative path."""
    rng = np.random.default_rng(seed)
    xs = rng.uniform(-1.5, 1.5, size=(N, 3)).astype(np.float32)
    trees = []
    for _ in range(M):
        K = int(rng.integers(K_lo, K_hi + 1))
        nodes = [("b", 1)] * (K - 1) + [("c",)]
        for k in range(1, K):
            v = int(rng.integers(3))
            kind = int(rng.integers(3))
            term = [("b", 3), ("c",)]
            if kind == 0:
                term += [("v", v)]
            elif kind == 1:
                term += [("u", 14), ("v", v)]
            else:
                term += [("b", 3), ("v", v), ("v", (v + 1) % 3)]
            nodes += term
        nt, nv, ci = make_tree(nodes)
        trees.append((nt, nv, ci, rng.normal(0, 1, K).astype(np.float32)))
    y = (np.sin(xs[:, 0]) + xs[:, 1] * xs[:, 2]).astype(np.float32)
    return popio.build_pop(trees, xs, y)


def test_blocks_large_k_path(co):
    """K in 17..32 uses the cooperative (per-warp Gram) accumulation."""
    pop = _sum_of_terms_pop(40, 17, 32, 700, seed=3)
    assert pop["K_max"] > 16
    _check_blocks(co, pop, "fp64", 1e-10)
    _check_blocks(co, pop, "fp32", 2e-4)


def test_blocks_long_trees_global_tape(co):
    """63-255-node trees: the reverse tape lives in global scratch (too large for shared
    memory next to a second resident block)."""
    pop = synth.make_config("long", M=24, N=600, seed=3)
    _check_blocks(co, pop, "fp64", 1e-9, max_cond=1e6)
    _check_values(co, pop, "fp64", 1e-12, U64, min_strict=0.8)


def test_blocks_per_tree_targets(co):
    pop = synth.make_config("physics", M=32, N=900, seed=1)
    _check_blocks(co, pop, "fp64", 1e-10)


def test_blocks_pop1000_reference_population(co):
    pop, _ = pop1000()
    _check_blocks(co, popio.slice_pop(pop, 200), "fp64", 1e-10)


def test_ragged_sample_counts(co):
    """N not a multiple of the block round, N = 1, N smaller than a warp."""
    for N in (1, 7, 33, 257, 513):
        pop = synth.make_config("pr1", M=20, N=N, seed=N)
        _check_values(co, pop, "fp64", 1e-12, U64, min_strict=0.9)
        _check_blocks(co, pop, "fp64", 1e-10)


def test_unknown_operator_is_zero(co):
    nt, nv, ci = make_tree([("b", 1), ("u", 99), ("v", 0), ("b", 77), ("c",), ("v", 0)])
    pop = popio.build_pop([(nt, nv, ci, [1.5])], np.array([[0.5], [2.0]], np.float32),
                          np.zeros((1, 2), np.float32))
    out = co.evaluate(pop, precision="fp64", values=True, jacobian=True)
    np.testing.assert_array_equal(out["values"][0], [0.0, 0.0])
    np.testing.assert_array_equal(out["jacobian"][0, 0], [0.0, 0.0])


def _fd_check(co, pop, precision, eps, rtol, min_frac):
    """The on-device finite-difference Jacobian (co_jacobian_fd) against the reverse-mode one
    (co_evaluate): two independent derivative paths of the same interpreter agree to the FD
    truncation error on well-scaled samples."""
    jr = co.evaluate(pop, precision=precision, values=False, jacobian=True)["jacobian"]
    jf = co.jacobian_fd(pop, precision=precision, eps=eps)
    Ks = np.asarray(pop["metas"])[:, 3]
    ok = tot = 0
    for m in range(int(pop["M"])):
        K = int(Ks[m])
        if K == 0:
            assert not np.any(jf[m])
            continue
        a, b = jf[m, :K], jr[m, :K]
        fin = np.isfinite(a) & np.isfinite(b)
        scale = np.maximum(np.abs(b), np.abs(b[fin]).max(initial=0) * 1e-3 + 1e-12)
        with np.errstate(all="ignore"):
            good = np.abs(a - b) <= rtol * scale
        ok += int(np.sum(good & fin))
        tot += int(fin.sum())
        assert not np.any(jf[m, K:]), m      # rows k >= K are never written
    assert ok / max(tot, 1) >= min_frac, ok / max(tot, 1)


def test_fd_jacobian_fp64_matches_reverse(co):
    _fd_check(co, synth.make_config("pr1", M=64, N=200, seed=3), "fp64", 1e-7, 1e-5, 0.97)


def test_fd_jacobian_fp64_matches_oracle_fd(co):
    """Same formula on the CPU (oracle.interp.fd_jacobian): the device FD columns agree to the
    conditioning of the difference quotient (an error e in f becomes 2e/h in J)."""
    pop = synth.make_config("pr1", M=48, N=150, seed=5)
    jf = co.jacobian_fd(pop, precision="fp64", eps=1e-6)
    strict = total = 0
    for m in range(int(pop["M"])):
        nt, nv, ci, _y, K = interp.tree_view(pop, m)
        if K == 0:
            continue
        off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][off:off + K], np.float64)
        ref = interp.fd_jacobian(nt, nv, ci, pop["xs"], c, 1e-6)
        S = interp.error_scale(nt, nv, ci, pop["xs"], c)
        h = np.maximum(np.abs(c) * 1e-6, 1e-300)
        for k in range(K):
            got = jf[m, k]
            tol = 1e-6 * np.abs(ref[:, k]) + 64 * U64 * 2 * (S + 1e-300) / h[k]
            both = np.isfinite(got) & np.isfinite(ref[:, k])
            with np.errstate(all="ignore"):
                ok = np.abs(got - ref[:, k]) <= tol
            assert np.all(ok[both]), (m, k)
            strict += int(np.sum(np.abs(got - ref[:, k])[both] <= 1e-6 * np.abs(ref[both, k]) + 1e-300))
            total += int(both.sum())
    assert strict / max(total, 1) >= 0.9


def test_fd_jacobian_fp32_reference_step(co):
    """fp32 with the reference's eps_rel = 1e-3 (batch_lm.cu:207): first-order truncation, so
    a loose tolerance; the point is the same column layout and step rule."""
    _fd_check(co, synth.make_config("pr1", M=64, N=200, seed=4), "fp32", 0.0, 2e-2, 0.9)


@pytest.fixture(scope="module")
def co_fwd():
    """A context whose evaluations use forward-mode tangents for K <= 2 (CUSR_EVAL_FWD=2 is
    read when the context is created)."""
    import os

    old = os.environ.get("CUSR_EVAL_FWD")
    os.environ["CUSR_EVAL_FWD"] = "2"
    try:
        c = InProcessCO(device_id=0)
    finally:
        if old is None:
            del os.environ["CUSR_EVAL_FWD"]
        else:
            os.environ["CUSR_EVAL_FWD"] = old
    yield c
    c.teardown()


def _small_k_pop(seed):
    """PR1 trees restricted to K <= 2 (the forward-mode classes) plus a few larger ones."""
    pop = synth.make_config("pr1", M=160, N=256, seed=seed)
    Ks = np.asarray(pop["metas"])[:, 3]
    idx = np.concatenate([np.flatnonzero(Ks <= 2), np.flatnonzero(Ks > 2)[:8]])
    return popio.slice_pop(pop, idx)


@pytest.mark.parametrize("precision,tol", [("fp64", 1e-10), ("fp32", 1e-3)])
def test_forward_mode_jacobian_matches_oracle(co_fwd, precision, tol):
    _check_jacobian(co_fwd, _small_k_pop(21), precision, tol)


def test_forward_mode_blocks_match_reverse(co, co_fwd):
    """Normal-equation blocks from forward tangents equal the reverse sweep's to rounding."""
    pop = _small_k_pop(22)
    a = co.evaluate(pop, precision="fp64", values=False, blocks=True)["blocks"]
    b = co_fwd.evaluate(pop, precision="fp64", values=False, blocks=True)["blocks"]
    for x, y in zip(a, b):
        fin = np.isfinite(x) & np.isfinite(y)
        assert np.array_equal(np.isfinite(x), np.isfinite(y))
        np.testing.assert_allclose(y[fin], x[fin], rtol=1e-11, atol=1e-11 * np.abs(x[fin]).max(initial=1.0))
