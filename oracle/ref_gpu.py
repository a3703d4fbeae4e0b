"""The reference's own CUDA LM path, run as a subprocess. TEST / BASELINE INFRASTRUCTURE ONLY.

`batch_lm_revad_prof` is cusr/kernel/batch_lm_revad.cu (reverse-mode AD Jacobian, host-driven
LM loop, fast-math fp32) built from the reference's sources for sm_100a with -DPROFILE by
oracle/Makefile (nothing is copied into this repository). Its PROFILE_JSON line carries
`loop_ms`, the LM-loop time the reference's own throughput figure is taken from:
trees/s = (M - K0 trees) / loop_ms (experiments/e6_kernel_sweep/sweep_e6.py:126-132).

The reference kernel implements only the strict operators: the benchmark grammar's log|x| and
sqrt|x| (LOOSE_LOG 21, LOOSE_SQRT 28 of cusr/benchmark/interp.py:30-34) are re-encoded as
LOG(ABS(x)) and SQRT(ABS(x)), the same functions with the same derivatives away from x = 0.
Its compile-time limits are checked before it runs (batch_lm_revad.cu:243-264, MAX_NODES 128;
int sample indexing needs M*N < 2^31, lm_core.cuh:124-141); a population beyond them is not
run.
"""
from __future__ import annotations

import json
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BINARY = HERE / "_ref" / "batch_lm_revad_prof"

UFUNC = 2
F_LOG, F_LOOSE_LOG, F_ABS, F_SQRT, F_LOOSE_SQRT = 20, 21, 26, 27, 28
LOOSE_UNSUPPORTED = (5, 7, 24)          # LOOSE_DIV, LOOSE_POW, LOOSE_INV
MAX_K, MAX_STACK, MAX_NODES = 32, 64, 128


def strict_ops(pop: dict) -> dict:
    """The population with LOOSE_LOG / LOOSE_SQRT nodes re-encoded as LOG / SQRT of ABS
    (one extra unary node each; constant ranks, c_init, xs and ym unchanged)."""
    M = int(pop["M"])
    metas = np.asarray(pop["metas"], np.int64).reshape(M, 4)
    nt_all, nv_all, ci_all = (np.asarray(pop[k]) for k in ("nt", "nv", "ci"))
    nts, nvs, cis, new_metas = [], [], [], []
    off = 0
    for m in range(M):
        o, n, c_off, K = (int(v) for v in metas[m])
        nt, nv, ci = nt_all[o:o + n], nv_all[o:o + n], ci_all[o:o + n]
        loose = (nt == UFUNC) & np.isin(nv.astype(np.int64), (F_LOOSE_LOG, F_LOOSE_SQRT))
        bad = (nt >= UFUNC) & np.isin(nv.astype(np.int64), LOOSE_UNSUPPORTED)
        if bad.any():
            raise ValueError(f"tree {m}: operator without a strict equivalent")
        if loose.any():
            rep = np.where(loose, 2, 1)
            pos = np.repeat(np.arange(n), rep)
            second = np.zeros(pos.size, bool)
            second[np.cumsum(rep) - 1] = loose          # the inserted ABS follows its operator
            nt2 = nt[pos].astype(np.int32)
            nv2 = nv[pos].astype(np.float32)
            ci2 = ci[pos].astype(np.int32)
            head = loose[pos] & ~second
            nv2[head & (nv[pos] == F_LOOSE_LOG)] = F_LOG
            nv2[head & (nv[pos] == F_LOOSE_SQRT)] = F_SQRT
            nv2[second] = F_ABS
            ci2[second] = -1
            nt, nv, ci = nt2, nv2, ci2
        nts.append(np.asarray(nt, np.int32))
        nvs.append(np.asarray(nv, np.float32))
        cis.append(np.asarray(ci, np.int32))
        new_metas.append((off, len(nts[-1]), c_off, K))
        off += len(nts[-1])
    out = dict(pop)
    out.update(nt=np.concatenate(nts), nv=np.concatenate(nvs), ci=np.concatenate(cis),
               metas=np.asarray(new_metas, np.int32).reshape(M, 4), total_nodes=off)
    return out


def within_limits(pop: dict) -> str | None:
    """None if the reference binary can run `pop`, else the limit it exceeds."""
    metas = np.asarray(pop["metas"]).reshape(-1, 4)
    if int(pop["K_max"]) > MAX_K:
        return f"K_max {pop['K_max']} > {MAX_K}"
    if int(pop["max_stack"]) > MAX_STACK:
        return f"max_stack {pop['max_stack']} > {MAX_STACK}"
    if metas.size and int(metas[:, 1].max()) > MAX_NODES:
        return f"a tree of {int(metas[:, 1].max())} nodes > MAX_NODES {MAX_NODES}"
    if int(pop["M"]) * int(pop["N"]) >= 2 ** 31:
        return "M*N >= 2^31 (int sample indexing)"
    return None


def _write_pop_bin(pop: dict, path: Path) -> None:
    """pop.bin v1 with the target row replicated per tree (the reference loader's layout)."""
    hdr = np.zeros(16, np.int32)
    hdr[:9] = (0x4D4C344D, 1, pop["M"], pop["total_nodes"], pop["total_c"], pop["N"],
               pop["n_vars"], pop["K_max"], pop["max_stack"])
    ym = np.asarray(pop["ym"], np.float32)
    if ym.ndim == 1:
        ym = np.broadcast_to(ym, (int(pop["M"]), int(pop["N"])))
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        for key, dt in (("nt", np.int32), ("nv", np.float32), ("ci", np.int32),
                        ("metas", np.int32), ("c_init", np.float32), ("xs", np.float32)):
            f.write(np.ascontiguousarray(pop[key], dt).tobytes())
        for m in range(int(pop["M"])):                  # row by row: no M x N temporary
            f.write(np.ascontiguousarray(ym[m]).tobytes())


class RefGPU:
    """One population written once; `run()` fits it with the reference binary and returns
    its outputs and PROFILE_JSON timings."""

    def __init__(self, pop: dict, binary: Path = BINARY, workdir: str | None = None):
        if not Path(binary).exists():
            raise FileNotFoundError(f"{binary} not built (make -C oracle)")
        self.binary = Path(binary)
        self.pop = strict_ops(pop)
        why = within_limits(self.pop)
        if why:
            raise ValueError(f"beyond the reference kernel's limits: {why}")
        self._tmp = tempfile.TemporaryDirectory(dir=workdir)
        self.dir = Path(self._tmp.name)
        self.path = self.dir / "pop.bin"
        _write_pop_bin(self.pop, self.path)
        metas = np.asarray(self.pop["metas"]).reshape(-1, 4)
        self.n_k0 = int(np.sum(metas[:, 3] == 0))

    def run(self, max_iter: int = 50, timeout_s: float = 600.0, device: int | None = None) -> dict:
        env = dict(os.environ)
        if device is not None:
            env["CUDA_VISIBLE_DEVICES"] = str(device)
        p = subprocess.run([str(self.binary), str(self.path), str(self.dir), "--max-iter",
                            str(int(max_iter)), "--quiet"], capture_output=True, text=True,
                           timeout=timeout_s, env=env)
        if p.returncode != 0:
            raise RuntimeError(f"reference binary exited {p.returncode}: {p.stderr[-2000:]}")
        prof = None
        for line in p.stdout.splitlines():
            if line.startswith("PROFILE_JSON "):
                prof = json.loads(line[len("PROFILE_JSON "):])
        if prof is None:
            raise RuntimeError("no PROFILE_JSON line from the reference binary")
        M = int(self.pop["M"])
        return {
            "profile": prof,
            "loop_ms": float(prof["loop_ms"]),
            "fits_per_s": (M - self.n_k0) / (float(prof["loop_ms"]) / 1e3),
            "status": np.fromfile(self.dir / "status.bin", np.int32),
            "c_final": np.fromfile(self.dir / "c_final.bin", np.float32),
            "loss_final": np.fromfile(self.dir / "loss_final.bin", np.float32),
            "loss_init": np.fromfile(self.dir / "loss_init.bin", np.float32),
        }

    def close(self) -> None:
        self._tmp.cleanup()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False
