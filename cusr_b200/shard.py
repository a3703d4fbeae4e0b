"""Expression sharding across GPUs: cost-balanced partition of a population and the gather
of per-shard fits back to one global result.

Trees are independent, so a population splits into shards with no exchange during the fit:
each process (one per GPU) fits its shard and the results are gathered to rank 0 in the
original tree order. Shards are balanced by estimated cost with the LPT rule (most expensive
tree first, onto the least-loaded shard).

The collective calls take a `torch.distributed` process group when one is initialised (NCCL
on the GPU box, gloo in the CPU tests); nothing here touches a GPU itself.
"""
from __future__ import annotations

import heapq

import numpy as np

from . import popio


def tree_costs(pop: dict) -> np.ndarray:
    """Estimated per-tree cost of one LM iteration: samples x (forward + reverse sweep over
    the tree's nodes + the normal-equation update over K(K+1)/2 entries)."""
    metas = np.asarray(pop["metas"], np.int64).reshape(-1, 4)
    n_nodes = metas[:, 1].astype(np.float64)
    K = metas[:, 3].astype(np.float64)
    return float(pop["N"]) * (2.0 * n_nodes + 0.5 * K * (K + 1) * 0.25 + 1.0)


def lpt_partition(costs, n_shards: int) -> list[np.ndarray]:
    """Indices of each shard (ascending), LPT greedy on `costs`. Deterministic."""
    costs = np.asarray(costs, np.float64)
    order = np.argsort(-costs, kind="stable")
    heap = [(0.0, s) for s in range(n_shards)]
    heapq.heapify(heap)
    parts: list[list[int]] = [[] for _ in range(n_shards)]
    for m in order:
        load, s = heapq.heappop(heap)
        parts[s].append(int(m))
        heapq.heappush(heap, (load + float(costs[m]), s))
    return [np.sort(np.asarray(p, np.int64)) for p in parts]


def shard(pop: dict, rank: int, world: int) -> tuple[dict, np.ndarray]:
    """(sub-population of `rank`, its tree indices in the global population)."""
    idx = lpt_partition(tree_costs(pop), world)[rank]
    return popio.slice_pop(pop, idx), idx


def merge(pop: dict, parts: list[tuple[np.ndarray, dict]]) -> dict:
    """Assemble per-shard results {c_final, status, loss_init, loss_final, iters} (each in its
    shard's own order) into global arrays in the population's tree order."""
    M = int(pop["M"])
    metas = np.asarray(pop["metas"], np.int64).reshape(-1, 4)
    out = dict(c_final=np.asarray(pop["c_init"], np.float64).copy(),
               status=np.zeros(M, np.int32), loss_init=np.zeros(M), loss_final=np.zeros(M),
               iters=np.zeros(M, np.int32))
    for idx, res in parts:
        off = 0
        for j, m in enumerate(idx):
            K = int(metas[m, 3])
            c_off = int(metas[m, 2])
            out["c_final"][c_off:c_off + K] = res["c_final"][off:off + K]
            off += K
            for key in ("status", "loss_init", "loss_final", "iters"):
                if key in res:
                    out[key][m] = res[key][j]
    return out


def gather_to_root(pop: dict, idx: np.ndarray, res: dict, group=None):
    """Gather every rank's (idx, result) to rank 0 over torch.distributed; rank 0 returns
    the merged global result, the other ranks return None."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    payload = (np.asarray(idx), {k: np.asarray(v) for k, v in res.items()})
    gathered = [None] * world if rank == 0 else None
    dist.gather_object(payload, gathered, dst=0, group=group)
    if rank != 0:
        return None
    return merge(pop, gathered)


def sample_range(N: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the contiguous sample slice of `rank` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    base, extra = divmod(int(N), int(world))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def sample_slice(pop: dict, rank: int, world: int) -> dict:
    """The population with only `rank`'s slice of the samples, for the sample-sharded mode
    (every rank keeps all trees and the same c_init; xs rows and ym columns are split)."""
    lo, hi = sample_range(int(pop["N"]), rank, world)
    out = dict(pop)
    out["xs"] = np.ascontiguousarray(np.asarray(pop["xs"], np.float32)[lo:hi])
    ym = np.asarray(pop["ym"], np.float32)
    out["ym"] = np.ascontiguousarray(ym[lo:hi] if ym.ndim == 1 else ym[:, lo:hi])
    out["N"] = hi - lo
    return out
