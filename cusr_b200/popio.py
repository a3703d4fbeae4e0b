"""pop.bin population files: read, write, build from trees, slice.

Byte format (cusr/kernel/pop_format.h:1-51, version 1, little-endian, no padding):
  header 16 x int32: magic, version, M, total_nodes, total_c, N, n_vars, K_max, max_stack, 0 x 7
  nt     int32[total_nodes]     node type (0 VAR, 1 CONST, 2 UFUNC, 3 BFUNC)
  nv     float32[total_nodes]   VAR -> variable index, FUNC -> operator id, CONST -> 0
  ci     int32[total_nodes]     CONST -> per-tree constant rank in prefix order, else -1
  metas  int32[M, 4]            (node_offset, n_nodes, c_offset, K)
  c_init float32[total_c]
  xs     float32[N, n_vars]
  ym     float32[M, N]

The in-memory pop dict uses the same keys as the reference loader
(cusr/benchmark/popio.py:26-41). `ym` may also be a single shared row of shape (N,) — the
extended entry point takes it without replicating it M times.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

POP_MAGIC = 0x4D4C344D
POP_VERSION = 1
NTYPE_VAR, NTYPE_CONST, NTYPE_UFUNC, NTYPE_BFUNC = 0, 1, 2, 3


def load_pop_bin(path) -> dict:
    with open(path, "rb") as f:
        hdr = struct.unpack("<16i", f.read(64))
        magic, version, M, total_n, total_c, N, n_vars, K_max, max_stack = hdr[:9]
        if magic != POP_MAGIC:
            raise ValueError(f"bad magic 0x{magic:08x} (want 0x{POP_MAGIC:08x})")
        if version != POP_VERSION:
            raise ValueError(f"pop.bin version {version} != {POP_VERSION}")

        def take(dtype, count):
            a = np.frombuffer(f.read(count * 4), dtype=dtype)
            if a.size != count:
                raise ValueError("short read")
            return a.copy()

        nt = take(np.int32, total_n)
        nv = take(np.float32, total_n)
        ci = take(np.int32, total_n)
        metas = take(np.int32, M * 4).reshape(M, 4)
        c_init = take(np.float32, total_c)
        xs = take(np.float32, N * n_vars).reshape(N, n_vars)
        ym = take(np.float32, M * N).reshape(M, N)
    return dict(M=M, total_nodes=total_n, total_c=total_c, N=N, n_vars=n_vars, K_max=K_max,
                max_stack=max_stack, nt=nt, nv=nv, ci=ci, metas=metas, c_init=c_init,
                xs=xs, ym=ym)


def save_pop_bin(pop: dict, path) -> None:
    hdr = np.zeros(16, np.int32)
    hdr[:9] = (POP_MAGIC, POP_VERSION, pop["M"], pop["total_nodes"], pop["total_c"], pop["N"],
               pop["n_vars"], pop["K_max"], pop["max_stack"])
    ym = np.asarray(pop["ym"], np.float32)
    if ym.ndim == 1:
        ym = np.broadcast_to(ym, (int(pop["M"]), int(pop["N"])))
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        for key, dt in (("nt", np.int32), ("nv", np.float32), ("ci", np.int32),
                        ("metas", np.int32), ("c_init", np.float32), ("xs", np.float32)):
            f.write(np.ascontiguousarray(pop[key], dt).tobytes())
        f.write(np.ascontiguousarray(ym).tobytes())


def stack_depth(nt) -> int:
    """Maximum evaluation-stack depth of a prefix tree evaluated right to left."""
    sp = best = 0
    for t in np.asarray(nt)[::-1]:
        t = int(t)
        if t in (NTYPE_VAR, NTYPE_CONST):
            sp += 1
        elif t == NTYPE_BFUNC:
            sp -= 1
        elif t != NTYPE_UFUNC:
            raise ValueError(f"unsupported node_type {t}")
        best = max(best, sp)
    return best


def build_pop(trees, xs, ym) -> dict:
    """trees = [(nt, nv, ci, c_init)], xs (N, n_vars), ym (M, N) or shared (N,) -> pop dict.
    Constant ranks must run 0..K-1 in prefix order (the reference invariant)."""
    xs = np.atleast_2d(np.asarray(xs, np.float32))
    nts, nvs, cis, metas, cs = [], [], [], [], []
    node_off = c_off = K_max = max_stack = 0
    for nt, nv, ci, c0 in trees:
        nt = np.asarray(nt, np.int32)
        ci = np.asarray(ci, np.int32)
        K = int(np.sum(nt == NTYPE_CONST))
        if [int(r) for r in ci[ci >= 0]] != list(range(K)):
            raise ValueError(f"constant ranks must be 0..{K - 1} in prefix order")
        c0 = np.asarray(c0, np.float32).ravel()
        if c0.size != K:
            raise ValueError(f"c_init has {c0.size} values, tree has K={K}")
        metas.append((node_off, len(nt), c_off, K))
        nts.append(nt)
        nvs.append(np.asarray(nv, np.float32))
        cis.append(ci)
        cs.append(c0)
        node_off += len(nt)
        c_off += K
        K_max = max(K_max, K)
        max_stack = max(max_stack, stack_depth(nt))
    ym = np.asarray(ym, np.float32)
    if ym.ndim != 1:
        ym = ym.reshape(len(trees), xs.shape[0])
    return dict(M=len(trees), total_nodes=node_off, total_c=c_off, N=xs.shape[0],
                n_vars=xs.shape[1], K_max=K_max, max_stack=max_stack,
                nt=np.concatenate(nts) if nts else np.zeros(0, np.int32),
                nv=np.concatenate(nvs) if nvs else np.zeros(0, np.float32),
                ci=np.concatenate(cis) if cis else np.zeros(0, np.int32),
                metas=np.asarray(metas, np.int32).reshape(-1, 4),
                c_init=np.concatenate(cs) if c_off else np.zeros(0, np.float32),
                xs=xs, ym=ym)


def tree_view(pop: dict, m: int):
    """(nt, nv, ci, y_row, K) of tree m."""
    off, n, _c_off, K = (int(v) for v in pop["metas"][m])
    ym = pop["ym"]
    y = ym if np.asarray(ym).ndim == 1 else ym[m]
    return pop["nt"][off:off + n], pop["nv"][off:off + n], pop["ci"][off:off + n], y, K


def tree_consts(pop: dict, c: np.ndarray, m: int) -> np.ndarray:
    _off, _n, c_off, K = (int(v) for v in pop["metas"][m])
    return c[c_off:c_off + K]


def slice_pop(pop: dict, idx) -> dict:
    """Sub-population of the trees `idx` (a limit int or an index array), offsets rebuilt."""
    if isinstance(idx, (int, np.integer)):
        idx = np.arange(min(int(idx), int(pop["M"])))
    idx = np.asarray(idx, np.int64)
    trees = []
    for m in idx:
        nt, nv, ci, _y, K = tree_view(pop, int(m))
        c_off = int(pop["metas"][m][2])
        trees.append((nt, nv, ci, pop["c_init"][c_off:c_off + K]))
    ym = pop["ym"]
    ym = ym if np.asarray(ym).ndim == 1 else np.asarray(ym)[idx]
    return build_pop(trees, pop["xs"], ym)


def replicate_ym(pop: dict) -> dict:
    """Copy of `pop` whose ym is the full [M, N] array (what the reference ABI expects)."""
    ym = np.asarray(pop["ym"], np.float32)
    if ym.ndim == 1:
        ym = np.ascontiguousarray(np.broadcast_to(ym, (int(pop["M"]), int(pop["N"]))))
    out = dict(pop)
    out["ym"] = ym
    return out


def _ranges(starts: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    """Concatenation of arange(s, s + n) for every (s, n) pair (vectorised)."""
    lengths = np.asarray(lengths, np.int64)
    total = int(lengths.sum())
    if total == 0:
        return np.zeros(0, np.int64)
    ends = np.cumsum(lengths)
    first = np.repeat(np.asarray(starts, np.int64) - (ends - lengths), lengths)
    return first + np.arange(total, dtype=np.int64)


def replicate(pop: dict, copies: int, c_init=None) -> dict:
    """Population whose tree j = m * copies + s is a copy of tree m (programs and targets);
    `c_init` (optional, [M * copies, ...] flattened in that order) replaces the constants.
    Shared-y populations stay shared; per-tree targets are repeated."""
    M, S = int(pop["M"]), int(copies)
    metas = np.asarray(pop["metas"], np.int64).reshape(M, 4)
    off, n, coff, K = metas[:, 0], metas[:, 1], metas[:, 2], metas[:, 3]
    n_r, K_r = np.repeat(n, S), np.repeat(K, S)
    node_idx = _ranges(np.repeat(off, S), n_r)
    c_idx = _ranges(np.repeat(coff, S), K_r)
    new_metas = np.stack([np.cumsum(n_r) - n_r, n_r, np.cumsum(K_r) - K_r, K_r], 1)
    ym = np.asarray(pop["ym"], np.float32)
    out = dict(pop)
    out.update(M=M * S, total_nodes=int(n_r.sum()), total_c=int(K_r.sum()),
               nt=np.asarray(pop["nt"], np.int32)[node_idx],
               nv=np.asarray(pop["nv"], np.float32)[node_idx],
               ci=np.asarray(pop["ci"], np.int32)[node_idx],
               metas=new_metas.astype(np.int32),
               c_init=(np.asarray(pop["c_init"], np.float32)[c_idx] if c_init is None
                       else np.asarray(c_init, np.float32).reshape(-1)),
               ym=ym if ym.ndim == 1 else np.repeat(ym, S, axis=0))
    if out["c_init"].size != out["total_c"]:
        raise ValueError("c_init does not match the replicated constants")
    return out
