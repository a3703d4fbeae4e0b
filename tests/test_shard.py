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
