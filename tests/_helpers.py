"""Shared test helpers: golden fixture loading, tolerance rules, tree construction."""
from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def report_dir() -> Path | None:
    """Directory for the measurement reports GPU tests write beside their assertions
    (parity fractions, error quantiles): CUSR_REPORT_DIR when set, else None (no report)."""
    d = os.environ.get("CUSR_REPORT_DIR")
    if not d:
        return None
    p = Path(d)
    p.mkdir(parents=True, exist_ok=True)
    return p


def write_report(name: str, data) -> None:
    """Write `data` as JSON to <report_dir>/<name> when a report directory is configured."""
    d = report_dir()
    if d is not None:
        (d / name).write_text(json.dumps(data, indent=1, default=float))

VAR, CONST, UFUNC, BFUNC = 0, 1, 2, 3


def load_npz_pop(z, prefix: str) -> dict:
    pop = {k: z[f"{prefix}/{k}"] for k in ("nt", "nv", "ci", "metas", "c_init", "xs", "ym")}
    for k in ("M", "total_nodes", "total_c", "N", "n_vars", "K_max", "max_stack"):
        pop[k] = int(z[f"{prefix}/{k}"])
    return pop


def fixture_pop(name: str) -> dict:
    z = np.load(GOLDEN / "fixtures.npz")
    pop = load_npz_pop(z, name)
    pop["loss_init64"] = z[f"{name}/loss_init64"]
    return pop


def fixture_truth(json_name: str) -> dict:
    return json.loads((GOLDEN / "fixtures.json").read_text())[json_name]


def pop1000() -> tuple[dict, dict]:
    z = np.load(GOLDEN / "pop1000.npz")
    pop = load_npz_pop(z, "pop")
    extra = {k: z[k] for k in z.files if not k.startswith("pop/")}
    return pop, extra


def conditioned_close(got, ref, scale, rel: float, unit: float, k: float = 64.0):
    """|got - ref| <= rel*|ref| + k*unit*scale elementwise (scale = oracle error_scale);
    both non-finite in the same way also counts as a match."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    both_nan = np.isnan(got) & np.isnan(ref)
    same_inf = np.isinf(got) & np.isinf(ref) & (np.sign(got) == np.sign(ref))
    with np.errstate(all="ignore"):
        ok = np.abs(got - ref) <= rel * np.abs(ref) + k * unit * np.asarray(scale, np.float64)
    return ok | both_nan | same_inf


def tree_consts(pop, c, m):
    off, K = int(pop["metas"][m][2]), int(pop["metas"][m][3])
    return np.asarray(c)[off:off + K]


def make_tree(nodes):
    """nodes: list of ('v', idx) / ('c',) / ('u', fid) / ('b', fid) in prefix order ->
    (nt, nv, ci) with constant ranks in prefix order."""
    nt, nv, ci = [], [], []
    k = 0
    for n in nodes:
        if n[0] == "v":
            nt.append(VAR); nv.append(float(n[1])); ci.append(-1)
        elif n[0] == "c":
            nt.append(CONST); nv.append(0.0); ci.append(k); k += 1
        elif n[0] == "u":
            nt.append(UFUNC); nv.append(float(n[1])); ci.append(-1)
        else:
            nt.append(BFUNC); nv.append(float(n[1])); ci.append(-1)
    return np.asarray(nt, np.int32), np.asarray(nv, np.float32), np.asarray(ci, np.int32)
