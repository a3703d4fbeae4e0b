"""Seeded synthetic populations for the benchmark configurations.

Every configuration is generated from `numpy.random.default_rng(seed)`, so the same
(name, M, N, seed) gives the same pop byte for byte. Trees are random prefix trees of the
reference bytecode (cusr/kernel/pop_format.h) with constant ranks in prefix order; a tree
whose value at its initial constants is non-finite or larger than 1e6 in magnitude on a check
subset of the samples is redrawn, as the reference's generator does
(cusr/benchmark/workload/gen_synth.py:136-140).

Configurations (shapes, sizes and value distributions of the benchmark plan):
  pr1      M=256    len 5-31    ops + - * / sin cos exp log|.| sqrt|.|  2 vars U[-3,3]
           K 1-6, c0 ~ N(0,1), N=1000, y = ground-truth tree + N(0, 0.01^2), fp64, 50 it
  mid      M=4096   len 7-63    same ops, 5 vars U[-5,5], K 1-12, N=10000,
           shared y = ground-truth tree + N(0, 0.05^2), fp32, 50 it
  metric   the mid generator with M=16384 (the headline metric's population)
  physics  M=1024   products / quotients / powers of 1-9 positive variables (x ~ logU[0.1,10])
           with one or two sin / exp / sqrt factors, K 1-8, per-tree y = tree(c_true) * (1 +
           0.01 eps), N=100000, fp64, 100 it
  long     M=16384  len 63-255, K 8-32, 3 vars U[-2,2], N=4096, shared y, fp32, 50 it
  scale    M=262144 len 5-127 (log-normal, median ~21), K 1-16, 4 vars U[-3,3], N=20000,
           shared y, fp32, 30 it
  sharded  M=512    the scale grammar at N=10,000,000, fp32, 30 it
"""
from __future__ import annotations

import numpy as np

from . import popio

VAR, CONST, UFUNC, BFUNC = 0, 1, 2, 3
ADD, SUB, MUL, DIV, POW = 1, 2, 3, 4, 6
SIN, COS, LOG, EXP, SQRT = 14, 15, 20, 22, 27
LOGABS, SQRTABS = 21, 28

BASE_BINARY = (ADD, SUB, MUL, DIV)
BASE_UNARY = (SIN, COS, EXP, LOGABS, SQRTABS)

CONFIGS = {
    "pr1": dict(M=256, N=1000, len=(5, 31), K=(1, 6), n_vars=2, x=("uniform", -3.0, 3.0),
                noise=0.01, precision="fp64", max_iter=50, unary_frac=0.3),
    "mid": dict(M=4096, N=10000, len=(7, 63), K=(1, 12), n_vars=5, x=("uniform", -5.0, 5.0),
                noise=0.05, precision="fp32", max_iter=50, unary_frac=0.3),
    "metric": dict(M=16384, N=10000, len=(7, 63), K=(1, 12), n_vars=5,
                   x=("uniform", -5.0, 5.0), noise=0.05, precision="fp32", max_iter=50,
                   unary_frac=0.3),
    "physics": dict(M=1024, N=100000, K=(1, 8), n_vars=9, x=("loguniform", 0.1, 10.0),
                    noise=0.01, precision="fp64", max_iter=100),
    "long": dict(M=16384, N=4096, len=(63, 255), K=(8, 32), n_vars=3, x=("uniform", -2.0, 2.0),
                 noise=0.05, precision="fp32", max_iter=50, unary_frac=0.2),
    "scale": dict(M=262144, N=20000, len=(5, 127), len_lognormal=(np.log(21.0), 0.6),
                  K=(1, 16), n_vars=4, x=("uniform", -3.0, 3.0), noise=0.05, precision="fp32",
                  max_iter=30, unary_frac=0.3),
    "sharded": dict(M=512, N=10_000_000, len=(5, 127), len_lognormal=(np.log(21.0), 0.6),
                    K=(1, 16), n_vars=4, x=("uniform", -3.0, 3.0), noise=0.05,
                    precision="fp32", max_iter=30, unary_frac=0.3),
}


# --------------------------------------------------------------------------- evaluation
def eval_tree(nt, nv, ci, xs, c) -> np.ndarray:
    """fp64 value of one prefix tree at every row of xs (right-to-left stack machine)."""
    xs = np.asarray(xs, np.float64)
    c = np.asarray(c, np.float64)
    st = []
    with np.errstate(all="ignore"):
        for i in range(len(nt) - 1, -1, -1):
            t = int(nt[i])
            if t == VAR:
                st.append(xs[:, int(nv[i])])
            elif t == CONST:
                st.append(np.full(xs.shape[0], c[int(ci[i])]))
            elif t == UFUNC:
                a = st.pop()
                f = int(nv[i])
                st.append({SIN: np.sin, COS: np.cos, EXP: np.exp, LOG: np.log,
                           SQRT: np.sqrt, LOGABS: lambda v: np.log(np.abs(v)),
                           SQRTABS: lambda v: np.sqrt(np.abs(v))}[f](a))
            else:
                l = st.pop()
                r = st.pop()
                f = int(nv[i])
                st.append({ADD: np.add, SUB: np.subtract, MUL: np.multiply, DIV: np.divide,
                           POW: np.power}[f](l, r))
    return st[0]


def _ok(y) -> bool:
    return bool(np.all(np.isfinite(y)) and np.max(np.abs(y)) <= 1e6)


# --------------------------------------------------------------------------- tree shapes
def _shape(rng, n: int, u: int, out: list) -> None:
    """Append node kinds ('L', 'U', 'B') of a random prefix tree with n nodes of which u are
    unary. Invariant: n - 1 - u is even and 0 <= u <= n - 1."""
    while True:
        if n == 1:
            out.append("L")
            return
        n_ops = (n - 1 + u) // 2
        if u > 0 and (u == n - 1 or rng.random() < u / n_ops):
            out.append("U")
            n, u = n - 1, u - 1
            continue
        out.append("B")
        while True:
            ls = int(rng.integers(1, n - 1))
            rs = n - 1 - ls
            lo, hi = max(0, u - (rs - 1)), min(ls - 1, u)
            if (lo - (ls - 1)) % 2:
                lo += 1
            if lo <= hi:
                break
        ul = lo + 2 * int(rng.integers(0, (hi - lo) // 2 + 1))
        _shape(rng, ls, ul, out)
        n, u = rs, u - ul


def _random_tree(rng, length: int, K: int, n_vars: int, unary_frac: float,
                 binary=BASE_BINARY, unary=BASE_UNARY):
    """Random prefix tree with exactly `length` nodes and K constants, or None."""
    u = int(round(unary_frac * (length - 1) / (2.0 - unary_frac)))
    if (u - (length - 1)) % 2:
        u += 1 if u < length - 1 else -1
    u = max(0, min(u, length - 1))
    while u >= 0 and (length - 1 - u) // 2 + 1 < K:
        u -= 2
    if u < 0 or (length - 1 - u) % 2:
        return None
    kinds: list = []
    _shape(rng, length, u, kinds)
    leaves = [i for i, k in enumerate(kinds) if k == "L"]
    if len(leaves) < K:
        return None
    const_pos = set(rng.choice(len(leaves), size=K, replace=False).tolist()) if K else set()
    nt = np.empty(length, np.int32)
    nv = np.zeros(length, np.float32)
    ci = np.full(length, -1, np.int32)
    rank = 0
    leaf_no = 0
    for i, k in enumerate(kinds):
        if k == "L":
            if leaf_no in const_pos:
                nt[i] = CONST
                ci[i] = rank
                rank += 1
            else:
                nt[i] = VAR
                nv[i] = float(rng.integers(n_vars)) if n_vars else 0.0
            leaf_no += 1
        elif k == "U":
            nt[i] = UFUNC
            nv[i] = float(unary[int(rng.integers(len(unary)))])
        else:
            nt[i] = BFUNC
            nv[i] = float(binary[int(rng.integers(len(binary)))])
    return nt, nv, ci


def _sample_len(rng, cfg) -> int:
    lo, hi = cfg["len"]
    if "len_lognormal" in cfg:
        mu, sig = cfg["len_lognormal"]
        return int(np.clip(round(rng.lognormal(mu, sig)), lo, hi))
    return int(rng.integers(lo, hi + 1))


def _inputs(rng, cfg, N: int) -> np.ndarray:
    kind, a, b = cfg["x"]
    n_vars = cfg["n_vars"]
    if kind == "uniform":
        return rng.uniform(a, b, size=(N, n_vars)).astype(np.float32)
    return np.exp(rng.uniform(np.log(a), np.log(b), size=(N, n_vars))).astype(np.float32)


def _grammar_pop(cfg, M: int, N: int, rng) -> dict:
    xs = _inputs(rng, cfg, N)
    chk = xs[: min(N, 512)]
    klo, khi = cfg["K"]
    # ground truth: one tree of the same grammar, constants ~ N(0, 1), shared by all trees
    while True:
        gt = _random_tree(rng, _sample_len(rng, cfg), int(rng.integers(klo, khi + 1)),
                          cfg["n_vars"], cfg["unary_frac"])
        if gt is None:
            continue
        c_gt = rng.standard_normal(int((gt[0] == CONST).sum()))
        y = eval_tree(*gt, xs, c_gt)
        if _ok(y) and (N < 2 or np.std(y) > 1e-6):
            break
    y = (y + cfg["noise"] * rng.standard_normal(N)).astype(np.float32)
    trees = []
    while len(trees) < M:
        K = int(rng.integers(klo, khi + 1))
        t = _random_tree(rng, _sample_len(rng, cfg), K, cfg["n_vars"], cfg["unary_frac"])
        if t is None:
            continue
        c0 = rng.standard_normal(K).astype(np.float32)
        if not _ok(eval_tree(*t, chk, c0)):
            continue
        trees.append((*t, c0))
    return popio.build_pop(trees, xs, y)


def _physics_tree(rng, n_vars: int, K_target: int):
    """c0 * prod x_v^(1 | -1 | c) * one or two of sin(c x), exp(c x), sqrt(c x)."""
    c_true: list = []   # constant values in prefix order

    def leaf_var(v):
        return [(VAR, float(v))]

    def leaf_const(val):
        c_true.append(val)
        return [(CONST, 0.0)]

    n_trans = 1 + int(rng.random() < 0.5)
    n_pow_budget = max(0, K_target - 1 - n_trans)
    n_fac = int(rng.integers(1, n_vars + 1))
    vars_ = rng.choice(n_vars, size=n_fac, replace=False)
    factors = []        # (op joining this factor: MUL or DIV, prefix node list builder)
    factors.append((MUL, lambda: leaf_const(float(rng.uniform(0.5, 3.0)))))
    for v in vars_:
        kind = rng.random()
        if n_pow_budget > 0 and kind < 0.4:
            n_pow_budget -= 1
            e = float(rng.uniform(0.5, 2.5) * rng.choice([-1.0, 1.0]))
            factors.append((MUL, lambda v=v, e=e: [(BFUNC, float(POW))] + leaf_var(v) + leaf_const(e)))
        elif kind < 0.7:
            factors.append((DIV, lambda v=v: leaf_var(v)))
        else:
            factors.append((MUL, lambda v=v: leaf_var(v)))
    for _ in range(n_trans):
        f = (SIN, EXP, SQRT)[int(rng.integers(3))]
        v = int(rng.integers(n_vars))
        cval = float(rng.uniform(0.1, 1.0))
        factors.append((MUL, lambda f=f, v=v, cval=cval:
                        [(UFUNC, float(f)), (BFUNC, float(MUL))] + leaf_const(cval) + leaf_var(v)))
    tail = factors[1:]
    rng.shuffle(tail)
    # left-deep chain (((f0 op1 f1) op2 f2) ... opn fn); its prefix form is
    # opn ... op1 f0 f1 ... fn
    out = [(BFUNC, float(op)) for op, _ in reversed(tail)]
    out += factors[0][1]()
    for _, build in tail:
        out += build()
    nt = np.array([t for t, _ in out], np.int32)
    nv = np.array([v for _, v in out], np.float32)
    ci = np.full(len(nt), -1, np.int32)
    ci[nt == CONST] = np.arange(int((nt == CONST).sum()), dtype=np.int32)
    return nt, nv, ci, np.asarray(c_true, np.float64)


def _physics_pop(cfg, M: int, N: int, rng) -> dict:
    xs = _inputs(rng, cfg, N)
    trees, ys, c_trues = [], [], []
    klo, khi = cfg["K"]
    while len(trees) < M:
        nt, nv, ci, c_true = _physics_tree(rng, cfg["n_vars"], int(rng.integers(klo, khi + 1)))
        K = int((nt == CONST).sum())
        if K < klo or K > khi:
            continue
        y = eval_tree(nt, nv, ci, xs, c_true)
        if not _ok(y):
            continue
        y = y * (1.0 + cfg["noise"] * rng.standard_normal(N))
        c0 = (c_true * rng.uniform(0.7, 1.3, K)).astype(np.float32)
        trees.append((nt, nv, ci, c0))
        ys.append(y.astype(np.float32))
        c_trues.append(c_true.astype(np.float32))
    pop = popio.build_pop(trees, xs, np.stack(ys))
    pop["c_true"] = np.concatenate(c_trues)
    return pop


def make_config(name: str, M: int | None = None, N: int | None = None, seed: int = 0) -> dict:
    """Generate configuration `name` (optionally resized). Adds 'name', 'precision',
    'max_iter' and 'seed' keys; shared targets are a 1-D ym row."""
    cfg = dict(CONFIGS[name])
    M = int(M if M is not None else cfg["M"])
    N = int(N if N is not None else cfg["N"])
    rng = np.random.default_rng(seed)
    pop = _physics_pop(cfg, M, N, rng) if name == "physics" else _grammar_pop(cfg, M, N, rng)
    pop.update(name=name, precision=cfg["precision"], max_iter=cfg["max_iter"], seed=seed)
    return pop
