"""co_evaluate_noalloc — the allocation-free evaluation entry, for callers that cannot
allocate device memory (their GPU memory belongs to their own pool allocator, or they cannot
take cudaMalloc's device-wide synchronisation inside their loop). It must give the same
normal-equation blocks as the allocating entry co_evaluate, call after call, although every
call reuses the one fixed scratch array inside the library.

Collected last on purpose (file name), so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _helpers import make_tree
from cusr_b200 import InProcessCO, co_inproc, popio, synth

pytestmark = pytest.mark.gpu

I32 = ctypes.POINTER(ctypes.c_int32)
F32 = ctypes.POINTER(ctypes.c_float)


def _bind():
    lib = ctypes.CDLL(str(co_inproc.default_lib_path()))
    fn = lib.co_evaluate_noalloc
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(co_inproc.PopHeader), I32, F32, I32,
                   ctypes.POINTER(co_inproc.TreeMeta), ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _call(fn, pop):
    """Call the entry point with device buffers the caller owns (allocated here by torch,
    sized for the population). Returns (rc, blocks)."""
    import torch

    dev = torch.device("cuda", 0)
    c = torch.as_tensor(np.asarray(pop["c_init"], np.float32), device=dev)
    xs = torch.as_tensor(np.ascontiguousarray(pop["xs"], np.float32), device=dev)
    y = torch.as_tensor(np.asarray(pop["ym"], np.float32).reshape(-1)[: pop["N"]], device=dev)
    Ks = pop["metas"][:, 3].astype(np.int64)
    n_out = int(np.sum((Ks + 1) * (Ks + 2) // 2))
    out = torch.full((max(n_out, 1),), float("nan"), dtype=torch.float32, device=dev)
    hdr = co_inproc.build_header(pop)
    nt = np.ascontiguousarray(pop["nt"], np.int32)
    nv = np.ascontiguousarray(pop["nv"], np.float32)
    ci = np.ascontiguousarray(pop["ci"], np.int32)
    metas = np.ascontiguousarray(pop["metas"], np.int32)
    torch.cuda.synchronize()
    rc = fn(0, ctypes.byref(hdr), nt.ctypes.data_as(I32), nv.ctypes.data_as(F32),
            ci.ctypes.data_as(I32), metas.ctypes.data_as(ctypes.POINTER(co_inproc.TreeMeta)),
            c.data_ptr(), xs.data_ptr(), y.data_ptr(), out.data_ptr(), None)
    torch.cuda.synchronize()
    return rc, out[:n_out].cpu().numpy().astype(np.float64)


def _noalloc_blocks(fn, pop):
    rc, blocks = _call(fn, pop)
    assert rc == co_inproc.CO_OK, rc
    return blocks


def _reference_blocks(pop):
    with InProcessCO(device_id=0) as co:
        parts = co.evaluate(pop, precision="fp32", values=False, blocks=True)["blocks"]
    return np.concatenate(parts)


def _assert_close(got, want):
    # the fp32 block tolerance of the evaluation tests: 2e-4 relative, with a floor of
    # 2e-4 * 1e-6 of the largest entry for entries that cancel to ~0
    fin = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), fin)
    tol = 2e-4 * (np.abs(want[fin]) + 1e-6 * np.max(np.abs(want[fin]), initial=0.0))
    assert np.all(np.abs(got[fin] - want[fin]) <= tol)


def test_noalloc_matches_evaluate_on_two_calls_in_a_row():
    fn = _bind()
    first = synth.make_config("mid", M=96, N=3000, seed=21)
    second = synth.make_config("pr1", M=40, N=700, seed=22)   # smaller: stale contents must not leak
    for pop in (first, second):
        _assert_close(_noalloc_blocks(fn, pop), _reference_blocks(pop))
    # and the same population twice gives the same bytes
    a = _noalloc_blocks(fn, second)
    b = _noalloc_blocks(fn, second)
    assert a.tobytes() == b.tobytes()


def test_noalloc_rejects_populations_beyond_the_fixed_array():
    fn = _bind()
    # 2,000,000 samples x 5 inputs: the transposed inputs alone exceed the 32 MiB array
    big = synth.make_config("mid", M=16, N=2_000_000, seed=23)
    rc, _ = _call(fn, big)
    assert rc == co_inproc.CO_ERR_BOUNDS


def test_noalloc_rejects_trees_whose_tape_needs_global_memory():
    """A tree whose reverse tape does not fit in shared memory beside a second resident block
    (the allocating entry would put it in a global-memory tape): CO_ERR_BOUNDS before any
    work is queued, and the caller's output buffer is left as it was."""
    fn = _bind()
    depth = 150                                   # sin(sin(...sin(c * x0)...)): 151 tape slots
    nodes = [("u", 14)] * depth + [("b", 3), ("c",), ("v", 0)]
    nt, nv, ci = make_tree(nodes)
    rng = np.random.default_rng(5)
    xs = rng.uniform(-1, 1, size=(512, 1)).astype(np.float32)
    pop = popio.build_pop([(nt, nv, ci, np.array([0.5], np.float32))], xs,
                          np.zeros(512, np.float32))
    rc, blocks = _call(fn, pop)
    assert rc == co_inproc.CO_ERR_BOUNDS
    assert np.all(np.isnan(blocks))
