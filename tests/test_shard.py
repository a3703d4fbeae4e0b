"""Expression sharding: LPT cost balance, merge, and the gather to rank 0 over a real
torch.distributed process group (gloo, world size 2, CPU)."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as tmp

from cusr_b200 import popio, shard, synth


def test_lpt_partition_covers_and_balances():
    pop = synth.make_config("mid", M=400, N=64, seed=1)
    costs = shard.tree_costs(pop)
    for n in (1, 2, 3, 8):
        parts = shard.lpt_partition(costs, n)
        allidx = np.sort(np.concatenate(parts))
        np.testing.assert_array_equal(allidx, np.arange(400))
        loads = np.array([costs[p].sum() for p in parts])
        assert loads.max() - loads.min() <= costs.max() + 1e-9


def test_merge_restores_global_order():
    pop = synth.make_config("pr1", M=50, N=16, seed=2)
    parts = shard.lpt_partition(shard.tree_costs(pop), 3)
    results = []
    for idx in parts:
        sub = popio.slice_pop(pop, idx)
        results.append((idx, {"c_final": sub["c_init"].astype(np.float64) + 1.0,
                              "status": np.asarray(idx, np.int32) % 5,
                              "loss_final": np.asarray(idx, np.float64),
                              "loss_init": np.zeros(len(idx)), "iters": np.ones(len(idx), np.int32)}))
    out = shard.merge(pop, results)
    np.testing.assert_allclose(out["c_final"], pop["c_init"].astype(np.float64) + 1.0)
    np.testing.assert_array_equal(out["status"], np.arange(50) % 5)
    np.testing.assert_array_equal(out["loss_final"], np.arange(50))


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pop = synth.make_config("pr1", M=37, N=8, seed=3)
    sub, idx = shard.shard(pop, rank, world)
    res = {"c_final": sub["c_init"].astype(np.float64) * 2.0,
           "status": np.full(len(idx), rank, np.int32), "loss_init": np.zeros(len(idx)),
           "loss_final": np.asarray(idx, np.float64), "iters": np.zeros(len(idx), np.int32)}
    out = shard.gather_to_root(pop, idx, res)
    if rank == 0:
        q.put((out["c_final"].tolist(), out["status"].tolist(), out["loss_final"].tolist()))
    dist.destroy_process_group()


def test_gather_to_root_gloo_world2():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    c, status, lf = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    pop = synth.make_config("pr1", M=37, N=8, seed=3)
    np.testing.assert_allclose(c, pop["c_init"].astype(np.float64) * 2.0)
    np.testing.assert_array_equal(lf, np.arange(37))
    parts = shard.lpt_partition(shard.tree_costs(pop), 2)
    for r, p in enumerate(parts):
        assert all(status[m] == r for m in p)


def test_sample_range_partitions():
    for N in (0, 1, 7, 10, 1001):
        for world in (1, 2, 3, 8):
            spans = [shard.sample_range(N, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def _normal_equations(pop):
    """Per tree: (JtJ, Jtr, 0.5 sum r^2) at c_init, fp64, from the oracle."""
    from oracle import interp

    out = []
    for m in range(int(pop["M"])):
        nt, nv, ci, y, K = interp.tree_view(pop, m)
        c_off = int(pop["metas"][m][2])
        c = np.asarray(pop["c_init"][c_off:c_off + K], np.float64)
        f, J = interp.value_and_jacobian(nt, nv, ci, pop["xs"], c)
        r = f - np.asarray(y, np.float64)
        out.append(np.concatenate([(J.T @ J)[np.triu_indices(K)], J.T @ r, [0.5 * r @ r]]))
    return np.concatenate(out)


def _sample_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pop = synth.make_config("pr1", M=24, N=301, seed=5)
    local = torch.from_numpy(_normal_equations(shard.sample_slice(pop, rank, world)))
    dist.all_reduce(local)          # the exchange step of the sample-sharded mode
    if rank == 0:
        q.put(local.numpy().tolist())
    dist.destroy_process_group()


def test_sample_sharded_normal_equations_gloo_world2():
    """Summing the per-slice normal equations over the group reproduces the full-sample
    ones: the decomposition the sample-sharded fit relies on."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sample_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    summed = np.asarray(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _normal_equations(synth.make_config("pr1", M=24, N=301, seed=5))
    finite = np.isfinite(full)
    np.testing.assert_array_equal(np.isfinite(summed), finite)
    np.testing.assert_allclose(summed[finite], full[finite], rtol=1e-10,
                               atol=1e-10 * np.abs(full[finite]).max())
