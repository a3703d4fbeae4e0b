"""In-process ctypes binding of libcusr_b200.so — the drop-in for CuSR's co_inproc module.

Same surface as the reference (cusr/kernel/co_inproc.py:29-295): `InProcessCO(device_id,
lib_path, variant).optimize(pop, max_iter)` returning {'c_final', 'status', 'loss_init',
'loss_final'}, the process-wide `get_inproc_co(device_id, variant)` singleton, `COError`
with the same return-code messages, and the `PopHeader` / `TreeMeta` ctypes mirrors.

Additions: `optimize_ex` (precision fp32 / fp64 / fp32_fast, shared targets, lambda0 /
xtol, Jacobian mode, robust damping, resident inputs across calls, fp64 outputs, per-tree
iteration counts), `load` / `fit_loaded` (population resident in HBM), `evaluate` and
`jacobian_fd` (one fused pass; finite-difference Jacobian), `shard_unique_id` /
`shard_init` / `optimize_sharded` (sample-sharded fits over NCCL) and `stats()` (phase
timings and work counters of the last call). There is no fallback path: if the shared
library is missing the constructor raises, and every fit runs on the GPU.
"""
from __future__ import annotations

import atexit
import ctypes
import threading
from pathlib import Path

import numpy as np

POP_MAGIC = 0x4D4C344D
POP_VERSION = 1

CO_OK = 0
CO_ERR_BOUNDS = 2
CO_ERR_CUDA = -1
CO_ERR_SUM_C = -2
CO_ERR_SUM_NODES = -3
CO_ERR_NULLARG = -4
CO_ERR_OOM = -5
CO_ERR_BADTREE = -6
SHARD_ID_BYTES = 128

CO_PREC_FP32 = 0
CO_PREC_FP64 = 1
CO_PREC_FP32_FAST = 2
# precision names: 'fp32' (IEEE fp32 functions), 'fp64', 'fp32_fast' (the reference kernel's
# --use_fast_math numerics)
PRECISIONS = {"fp32": CO_PREC_FP32, "fp64": CO_PREC_FP64, "fp32_fast": CO_PREC_FP32_FAST}


AD_MODES = {"auto": 0, "forward": 1, "reverse": 2}
# LM algorithm: the reference schedule (co_lib.cu) or MINPACK's trust region (the reference's
# scipy backend)
ALGORITHMS = {"reference": 0, "trust_region": 1}


def prec_code(precision: str) -> int:
    try:
        return PRECISIONS[precision]
    except KeyError:
        raise ValueError(f"precision must be one of {sorted(PRECISIONS)}") from None

STATUS_CONVERGED, STATUS_MAXITER, STATUS_FAIL_NAN, STATUS_K0_SKIP, STATUS_FAIL_CHOLESKY = range(5)

_ERR_MSG = {
    CO_ERR_BOUNDS: "K_max > MAX_K(32) or max_stack > MAX_STACK(64) (caller must pre-filter)",
    CO_ERR_CUDA: "CUDA error inside co_optimize",
    CO_ERR_SUM_C: "sum(metas.K) != header.total_c (pop inconsistent)",
    CO_ERR_SUM_NODES: "sum(metas.n_nodes) != header.total_nodes (pop inconsistent)",
    CO_ERR_NULLARG: "null pointer / bad argument",
    CO_ERR_OOM: "out of memory growing a device buffer",
    CO_ERR_BADTREE: "malformed tree bytecode (node type, stack, var index or const rank)",
}


class COError(RuntimeError):
    """Raised when co_init / co_optimize returns a non-OK code."""

    def __init__(self, code: int, where: str):
        self.code = code
        msg = _ERR_MSG.get(code, f"unknown code {code}")
        super().__init__(f"{where}: {msg} (code={code})")


class PopHeader(ctypes.Structure):
    _fields_ = [
        ("magic", ctypes.c_int32), ("version", ctypes.c_int32), ("M_prob", ctypes.c_int32),
        ("total_nodes", ctypes.c_int32), ("total_c", ctypes.c_int32), ("N", ctypes.c_int32),
        ("n_vars", ctypes.c_int32), ("K_max", ctypes.c_int32), ("max_stack", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 7),
    ]


class TreeMeta(ctypes.Structure):
    _fields_ = [("node_offset", ctypes.c_int32), ("n_nodes", ctypes.c_int32),
                ("c_offset", ctypes.c_int32), ("K", ctypes.c_int32)]


class CoOptions(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_int32), ("precision", ctypes.c_int32),
        ("max_iter", ctypes.c_int32), ("y_shared", ctypes.c_int32),
        ("lambda0", ctypes.c_double), ("xtol", ctypes.c_double),
        ("fp64_audit", ctypes.c_int32), ("early_exit", ctypes.c_int32),
        ("sample_sharded", ctypes.c_int32), ("keep_inputs", ctypes.c_int32),
        ("ad_mode", ctypes.c_int32), ("damping_always", ctypes.c_int32),
        ("damping_floor", ctypes.c_double),
        ("algorithm", ctypes.c_int32), ("n_starts", ctypes.c_int32),
        ("tr_starts", ctypes.c_int32), ("wave1", ctypes.c_int32),
        ("ftol", ctypes.c_double), ("gtol", ctypes.c_double), ("agree_tol", ctypes.c_double),
        ("start_seed", ctypes.c_uint64), ("fd_ordering", ctypes.c_int32),
        ("n_devices", ctypes.c_int32), ("device_ids", ctypes.c_int32 * 8),
        ("tr_dd", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class CoStats(ctypes.Structure):
    _fields_ = [
        ("setup_ms", ctypes.c_double), ("loop_ms", ctypes.c_double),
        ("finish_ms", ctypes.c_double), ("eval_ms", ctypes.c_double),
        ("step_ms", ctypes.c_double), ("device_ms", ctypes.c_double),
        ("flops", ctypes.c_double), ("node_evals", ctypes.c_int64), ("sample_evals", ctypes.c_int64),
        ("eval_launches", ctypes.c_int64), ("kernel_launches", ctypes.c_int64),
        ("iters_run", ctypes.c_int32), ("n_bins", ctypes.c_int32),
        ("y_shared", ctypes.c_int32), ("precision", ctypes.c_int32),
        ("n_reverted", ctypes.c_int32), ("n_starts", ctypes.c_int32),
        ("fits_run", ctypes.c_int64), ("trees_retired", ctypes.c_int32),
        ("reserved", ctypes.c_int32), ("comm_ms", ctypes.c_double),
    ]


assert ctypes.sizeof(PopHeader) == 64
assert ctypes.sizeof(TreeMeta) == 16

_F32 = ctypes.POINTER(ctypes.c_float)
_F64 = ctypes.POINTER(ctypes.c_double)
_I32 = ctypes.POINTER(ctypes.c_int32)

_HERE = Path(__file__).resolve().parent
LIB_NAME = "libcusr_b200.so"

# Every symbol include/cusr_co.h declares, with its ctypes signature.
SIGNATURES = {
    "co_init": ([ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "co_optimize": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                     ctypes.POINTER(TreeMeta), _F32, _F32, _F32, ctypes.c_int,
                     _F32, _I32, _F32, _F32], ctypes.c_int),
    "co_last_split": ([ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)],
                      ctypes.c_int),
    "co_teardown": ([ctypes.c_void_p], None),
    "co_default_options": ([ctypes.POINTER(CoOptions)], None),
    "co_optimize_ex": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                        ctypes.POINTER(TreeMeta), _F32, _F32, _F32,
                        ctypes.POINTER(CoOptions), _F64, _I32, _F64, _F64, _I32], ctypes.c_int),
    "co_get_stats": ([ctypes.c_void_p, ctypes.POINTER(CoStats)], ctypes.c_int),
    "co_strerror": ([ctypes.c_int], ctypes.c_char_p),
    "co_probe_peak": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_double),
                       ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "co_load": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                 ctypes.POINTER(TreeMeta), _F32, _F32, _F32, ctypes.POINTER(CoOptions)],
                ctypes.c_int),
    "co_fit_loaded": ([ctypes.c_void_p, ctypes.POINTER(CoOptions), _F64, _I32, _F64, _F64, _I32],
                      ctypes.c_int),
    "co_evaluate": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                     ctypes.POINTER(TreeMeta), _F64, _F32, _F32, ctypes.c_int, ctypes.c_int,
                     _F64, _F64, _F64], ctypes.c_int),
    "co_jacobian_fd": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                        ctypes.POINTER(TreeMeta), _F64, _F32, _F32, ctypes.c_int, ctypes.c_int,
                        ctypes.c_double, _F64], ctypes.c_int),
    "co_last_starts": ([ctypes.c_void_p, _I32], ctypes.c_int),
    "co_shard_unique_id": ([ctypes.POINTER(ctypes.c_ubyte)], ctypes.c_int),
    "co_shard_init": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_ubyte), ctypes.c_int,
                       ctypes.c_int, ctypes.c_double], ctypes.c_int),
    "co_optimize_sharded": ([ctypes.c_void_p, ctypes.POINTER(PopHeader), _I32, _F32, _I32,
                             ctypes.POINTER(TreeMeta), _F32, _F32, _F32,
                             ctypes.POINTER(CoOptions), _F64, _I32, _F64, _F64, _I32],
                            ctypes.c_int),
}


def default_lib_path() -> Path:
    return _HERE / LIB_NAME


def load_library(lib_path: str | Path | None = None) -> ctypes.CDLL:
    """Load the engine library and bind every exported C-ABI symbol."""
    path = Path(lib_path) if lib_path else default_lib_path()
    if not path.exists():
        raise FileNotFoundError(
            f"{path} is not built; run `python -m cusr_b200.build` (needs nvcc)")
    lib = ctypes.CDLL(str(path.resolve()))
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


def shard_unique_id(lib_path: str | Path | None = None) -> bytes:
    """A new 128-byte group id for the sample-sharded mode (co_shard_unique_id); create it
    on one rank and give it to every rank's InProcessCO.shard_init."""
    lib = load_library(lib_path)
    buf = (ctypes.c_ubyte * SHARD_ID_BYTES)()
    rc = lib.co_shard_unique_id(buf)
    if rc != CO_OK:
        raise COError(rc, "co_shard_unique_id")
    return bytes(buf)


def _c_ptr(arr, dtype):
    a = np.ascontiguousarray(arr, dtype=dtype)
    return a.ctypes.data_as(ctypes.POINTER(np.ctypeslib.as_ctypes_type(dtype))), a


def build_header(pop: dict) -> PopHeader:
    """Full 64-byte header from a pop dict (key 'M', no magic/version)."""
    h = PopHeader()
    h.magic = POP_MAGIC
    h.version = POP_VERSION
    h.M_prob = int(pop["M"])
    h.total_nodes = int(pop["total_nodes"])
    h.total_c = int(pop["total_c"])
    h.N = int(pop["N"])
    h.n_vars = int(pop["n_vars"])
    h.K_max = int(pop["K_max"])
    h.max_stack = int(pop["max_stack"])
    for i in range(7):
        h.reserved[i] = 0
    return h


def start_options(opt: CoOptions, algorithm: str = "reference", n_starts: int = 1,
                  tr_starts: int = 0, wave1: int = 0, ftol: float = 1e-10, gtol: float = 1e-8,
                  agree_tol: float = 1e-7, seed: int = 0, tr_dd: bool = False) -> CoOptions:
    """Fill the algorithm / start-axis fields of `opt`:
      algorithm  'reference' (the reference LM schedule) | 'trust_region' (MINPACK lmder: max_iter
                 then counts function evaluations, the first included, like scipy's max_nfev)
      n_starts   fits per tree (start 0 = c_init; the others generated on the device)
      tr_starts  > 0: starts 0..tr_starts-1 use the trust region, the others the reference
                 schedule (alternately with the floored damping on every solve)
      wave1      0 < wave1 < n_starts: run starts 0..wave1-1 first, then the rest only for trees
                 whose first-wave fits do not agree within agree_tol
      ftol, gtol trust-region tolerances; seed: start points
      tr_dd      trust-region fits (fp64) with double-double normal equations"""
    try:
        opt.algorithm = ALGORITHMS[algorithm]
    except KeyError:
        raise ValueError(f"algorithm must be one of {sorted(ALGORITHMS)}") from None
    opt.n_starts = int(n_starts)
    opt.tr_starts = int(tr_starts)
    opt.wave1 = int(wave1)
    opt.ftol = float(ftol)
    opt.gtol = float(gtol)
    opt.agree_tol = float(agree_tol)
    opt.start_seed = int(seed) & (2 ** 64 - 1)
    opt.tr_dd = 1 if tr_dd else 0
    return opt


# The parity-grade fit, in two device calls: every tree's 128 starts explored at once with the
# trust-region LM of the reference's scipy backend in fp32 (30 evaluations, ftol = xtol = 1e-6,
# two waves: trees whose first 8 fits agree skip the rest), then each tree's best fit polished
# in fp64 with scipy's tolerances (100 evaluations) from 8 starts around it (the best itself
# and 7 perturbations of it, one wave); the lower final loss is kept. Measured on the eight
# scipy samples (about 800 trees): 9 trees not within 1e-6 of the reference fit (the same with
# 60 or 200 polish evaluations), as for 50 exploration evaluations and a 16-start polish at
# twice the device time, and 8 for 96 fp64 starts (PARITY_FP64) at about five times it.
PARITY = dict(precision="fp64", max_iter=200, xtol=1e-10, damping_floor=1e-3,
              algorithm="trust_region", n_starts=128, tr_starts=128, wave1=8, ftol=1e-10,
              gtol=1e-8, polish=True, explore_precision="fp32", explore_max_iter=30,
              explore_tol=1e-6, polish_starts=8, polish_max_iter=100, dd_starts=0)

# 50 exploration evaluations and a single-start polish: 11-12 of about 800 trees off the
# reference fit, the lowest device time.
PARITY_FAST = dict(PARITY, explore_max_iter=50, polish_starts=1, polish_max_iter=200)

# PARITY and a third call: 16 fp64 trust-region starts from c_init on double-double normal
# equations (CoOptions.tr_dd). On the eight scipy samples 5 trees off the reference fit
# (PARITY 9) at about three times PARITY's device time.
PARITY_MAX = dict(PARITY, dd_starts=16)

# Every stage in fp64: 96 trust-region starts (200 evaluations, scipy's tolerances), then a
# single-start polish of each tree's best.
PARITY_FP64 = dict(precision="fp64", max_iter=200, xtol=1e-10, damping_floor=1e-3,
                   algorithm="trust_region", n_starts=96, tr_starts=96, wave1=8, ftol=1e-10,
                   gtol=1e-8, polish=True, explore_precision=None, explore_max_iter=None,
                   explore_tol=None, polish_starts=1, polish_max_iter=None, dd_starts=0)


class InProcessCO:
    """One persistent engine context on one device. CUDA context creation is paid once in
    __init__; every optimize() starts from the pop's c_init."""

    def __init__(self, device_id: int = 0, lib_path: str | None = None, variant: str = "ad"):
        self.variant = variant
        self.device_id = int(device_id)
        self._lib = load_library(lib_path)
        self._handle = ctypes.c_void_p()
        self._torn = False
        rc = self._lib.co_init(self.device_id, ctypes.byref(self._handle))
        if rc != CO_OK:
            raise COError(rc, "co_init")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.teardown()
        return False

    _build_header = staticmethod(build_header)

    def _inputs(self, pop: dict, y_shared: bool = False, keep_inputs: bool = False):
        M = int(pop["M"])
        keep = []

        def ptr(key, dtype):
            p, a = _c_ptr(pop[key], dtype)
            keep.append(a)
            return p

        if keep_inputs:   # X / y stay resident on the device: no pointers passed
            metas_buf = self._metas(pop, keep)
            return (ptr("nt", np.int32), ptr("nv", np.float32), ptr("ci", np.int32), metas_buf,
                    ptr("c_init", np.float32), None, None), keep
        ym = np.asarray(pop["ym"], np.float32)
        if y_shared:
            ym = ym.reshape(-1)[: int(pop["N"])]
        elif ym.ndim == 1:
            # the reference ABI takes [M][N] targets: replicate a shared row
            ym = np.broadcast_to(ym, (M, int(pop["N"])))
        ym_p, ym_a = _c_ptr(ym, np.float32)
        keep.append(ym_a)
        metas_buf = self._metas(pop, keep)
        return (ptr("nt", np.int32), ptr("nv", np.float32), ptr("ci", np.int32), metas_buf,
                ptr("c_init", np.float32), ptr("xs", np.float32), ym_p), keep

    @staticmethod
    def _metas(pop: dict, keep: list):
        M = int(pop["M"])
        metas_np = np.ascontiguousarray(pop["metas"], dtype=np.int32).reshape(M, 4)
        metas_buf = (TreeMeta * max(M, 1))()
        if M:
            ctypes.memmove(metas_buf, metas_np.ctypes.data, M * 16)
        keep.append(metas_buf)
        return metas_buf

    def optimize(self, pop: dict, max_iter: int = 50):
        """Reference-compatible fit (fp32). Returns {'c_final','status','loss_init',
        'loss_final'} sliced to this pop's sizes; raises COError on a non-OK code."""
        if self._torn:
            raise RuntimeError("InProcessCO used after teardown()")
        M, total_c = int(pop["M"]), int(pop["total_c"])
        hdr = build_header(pop)
        args, keep = self._inputs(pop)
        c_final = np.zeros(total_c, np.float32)
        status = np.zeros(M, np.int32)
        loss_init = np.zeros(M, np.float32)
        loss_final = np.zeros(M, np.float32)
        rc = self._lib.co_optimize(
            self._handle, ctypes.byref(hdr), *args, int(max_iter),
            c_final.ctypes.data_as(_F32), status.ctypes.data_as(_I32),
            loss_init.ctypes.data_as(_F32), loss_final.ctypes.data_as(_F32))
        del keep
        if rc != CO_OK:
            raise COError(rc, "co_optimize")
        out = {"c_final": c_final, "status": status}
        if self.variant == "ad":
            out["loss_init"] = loss_init
            out["loss_final"] = loss_final
        return out

    def optimize_ex(self, pop: dict, max_iter: int = 50, precision: str = "fp32",
                    y_shared: bool | None = None, lambda0: float = 1e-3, xtol: float = 1e-6,
                    fp64_audit: int = -1, early_exit: bool = True, keep_inputs: bool = False,
                    ad_mode: str = "auto", damping_floor: float = 0.0,
                    damping_always: bool = False, devices=None, **starts):
        """Extended fit: precision 'fp32' | 'fp64' | 'fp32_fast'; y_shared=True passes one
        target row (pop['ym'] may then be (N,) or (M, N) with identical rows; None = auto: a
        1-D ym). keep_inputs=True reuses the X / shared y left on the device by the previous
        call (pop needs no 'xs' / 'ym' then): the in-loop case of new trees on fixed data.
        ad_mode 'auto' | 'forward' (tangents for K <= 2) | 'reverse'. damping_floor > 0
        retries a system the reference damping diag*(1+lam) cannot factor with
        diag + lam*max(diag, f*max diag) (damping_always: use that damping on every solve).
        `starts` (see start_options): algorithm 'reference' | 'trust_region', n_starts,
        tr_starts, wave1, ftol, gtol, agree_tol, seed. devices=[d0, d1, ...] (up to 8): the
        trees are split into cost-balanced shards fitted concurrently on those devices in this
        one call (CoOptions.n_devices / device_ids).
        Returns fp64 c_final / loss_init / loss_final plus status and per-tree iters (and,
        with n_starts > 1, 'start': the start each tree's outputs came from)."""
        if devices is not None:
            starts = dict(starts, devices=list(devices))
        return self._fit_ex("co_optimize_ex", pop, max_iter, precision, y_shared, lambda0,
                            xtol, fp64_audit, early_exit, keep_inputs, ad_mode, damping_floor,
                            damping_always, starts)

    def shard_init(self, unique_id: bytes, nranks: int, rank: int,
                   timeout_s: float = 120.0) -> None:
        """Join a sample-sharded group (co_shard_init). `unique_id` comes from
        shard_unique_id() on one rank, shared with the others (e.g. a torch.distributed
        broadcast). Every later wait of a sharded fit is bounded by `timeout_s`."""
        if len(unique_id) != SHARD_ID_BYTES:
            raise ValueError(f"unique id must be {SHARD_ID_BYTES} bytes")
        buf = (ctypes.c_ubyte * SHARD_ID_BYTES).from_buffer_copy(unique_id)
        rc = self._lib.co_shard_init(self._handle, buf, int(nranks), int(rank), float(timeout_s))
        if rc != CO_OK:
            raise COError(rc, "co_shard_init")

    def optimize_sharded(self, pop: dict, max_iter: int = 50, precision: str = "fp32",
                         y_shared: bool | None = None, lambda0: float = 1e-3,
                         xtol: float = 1e-6, fp64_audit: int = -1, early_exit: bool = True,
                         keep_inputs: bool = False):
        """Sample-sharded fit (co_optimize_sharded): `pop` carries the whole population but
        only this rank's slice of the samples (pop['N'], 'xs', 'ym'); the normal equations
        are summed over the group every iteration, so every rank returns the same result."""
        return self._fit_ex("co_optimize_sharded", pop, max_iter, precision, y_shared, lambda0,
                            xtol, fp64_audit, early_exit, keep_inputs)

    def _fit_ex(self, entry, pop, max_iter, precision, y_shared, lambda0, xtol, fp64_audit,
                early_exit, keep_inputs=False, ad_mode="auto", damping_floor=0.0,
                damping_always=False, starts=None):
        if self._torn:
            raise RuntimeError("InProcessCO used after teardown()")
        M, total_c = int(pop["M"]), int(pop["total_c"])
        if keep_inputs:
            y_shared = True
        elif y_shared is None:
            y_shared = np.asarray(pop["ym"]).ndim == 1
        hdr = build_header(pop)
        args, keep = self._inputs(pop, y_shared=bool(y_shared), keep_inputs=keep_inputs)
        opt = self._options(max_iter, precision, y_shared, lambda0, xtol, fp64_audit, early_exit,
                            ad_mode)
        opt.keep_inputs = 1 if keep_inputs else 0
        opt.damping_floor = float(damping_floor)
        opt.damping_always = 1 if damping_always else 0
        starts = dict(starts or {})
        devices = starts.pop("devices", None)
        start_options(opt, **starts)
        if devices:
            if len(devices) > len(opt.device_ids):
                raise ValueError(f"at most {len(opt.device_ids)} devices per call")
            opt.n_devices = len(devices)
            for i, d in enumerate(devices):
                opt.device_ids[i] = int(d)
        c_final = np.zeros(total_c, np.float64)
        status = np.zeros(M, np.int32)
        loss_init = np.zeros(M, np.float64)
        loss_final = np.zeros(M, np.float64)
        iters = np.zeros(M, np.int32)
        rc = getattr(self._lib, entry)(
            self._handle, ctypes.byref(hdr), *args, ctypes.byref(opt),
            c_final.ctypes.data_as(_F64), status.ctypes.data_as(_I32),
            loss_init.ctypes.data_as(_F64), loss_final.ctypes.data_as(_F64),
            iters.ctypes.data_as(_I32))
        del keep
        if rc != CO_OK:
            raise COError(rc, entry)
        out = {"c_final": c_final, "status": status, "loss_init": loss_init,
               "loss_final": loss_final, "iters": iters}
        if opt.n_starts > 1:
            out["start"] = self.last_starts(M)
        return out

    def _options(self, max_iter=50, precision="fp32", y_shared=False, lambda0=1e-3, xtol=1e-6,
                 fp64_audit=-1, early_exit=True, ad_mode="auto") -> CoOptions:
        opt = CoOptions()
        self._lib.co_default_options(ctypes.byref(opt))
        opt.ad_mode = AD_MODES[ad_mode]
        opt.precision = prec_code(precision)
        opt.max_iter = int(max_iter)
        opt.y_shared = 1 if y_shared else 0
        opt.lambda0 = float(lambda0)
        opt.xtol = float(xtol)
        opt.fp64_audit = int(fp64_audit)
        opt.early_exit = 1 if early_exit else 0
        return opt

    def load(self, pop: dict, precision: str = "fp32", y_shared: bool | None = None,
             ad_mode: str = "auto", n_starts: int = 1) -> None:
        """Upload a population once (co_load); fit it with fit_loaded() any number of times.
        ad_mode fixes the Jacobian mode of the loaded schedule, n_starts the fits per tree."""
        if y_shared is None:
            y_shared = np.asarray(pop["ym"]).ndim == 1
        hdr = build_header(pop)
        args, keep = self._inputs(pop, y_shared=bool(y_shared))
        opt = self._options(precision=precision, y_shared=y_shared, ad_mode=ad_mode)
        opt.n_starts = int(n_starts)
        rc = self._lib.co_load(self._handle, ctypes.byref(hdr), *args, ctypes.byref(opt))
        del keep
        if rc != CO_OK:
            raise COError(rc, "co_load")
        self._loaded = (int(pop["M"]), int(pop["total_c"]), precision, int(n_starts))

    def fit_loaded(self, max_iter: int = 50, lambda0: float = 1e-3, xtol: float = 1e-6,
                   fp64_audit: int = -1, early_exit: bool = True,
                   sample_sharded: bool = False, precision: str | None = None,
                   damping_floor: float = 0.0, **starts) -> dict:
        """LM fit of the resident population from its c_init (inputs already in HBM).
        sample_sharded=True: the loaded samples are this rank's slice and the normal
        equations are summed over the shard_init group each iteration. `precision` may switch
        between 'fp32' and 'fp32_fast' on an fp32 load (default: the load's). `starts` as in
        optimize_ex (n_starts is the load's)."""
        M, total_c, loaded_prec, n_starts = self._loaded
        precision = precision or loaded_prec
        opt = self._options(max_iter, precision, False, lambda0, xtol, fp64_audit, early_exit)
        opt.sample_sharded = 1 if sample_sharded else 0
        opt.damping_floor = float(damping_floor)
        start_options(opt, **starts)
        opt.n_starts = n_starts
        c_final = np.zeros(total_c, np.float64)
        status = np.zeros(M, np.int32)
        loss_init = np.zeros(M, np.float64)
        loss_final = np.zeros(M, np.float64)
        iters = np.zeros(M, np.int32)
        rc = self._lib.co_fit_loaded(
            self._handle, ctypes.byref(opt), c_final.ctypes.data_as(_F64),
            status.ctypes.data_as(_I32), loss_init.ctypes.data_as(_F64),
            loss_final.ctypes.data_as(_F64), iters.ctypes.data_as(_I32))
        if rc != CO_OK:
            raise COError(rc, "co_fit_loaded")
        out = {"c_final": c_final, "status": status, "loss_init": loss_init,
               "loss_final": loss_final, "iters": iters}
        if n_starts > 1:
            out["start"] = self.last_starts(M)
        return out

    def last_starts(self, M: int) -> np.ndarray:
        """The start each tree's outputs of the last fit came from (co_last_starts)."""
        out = np.zeros(max(int(M), 1), np.int32)
        rc = self._lib.co_last_starts(self._handle, out.ctypes.data_as(_I32))
        if rc != CO_OK:
            raise COError(rc, "co_last_starts")
        return out[:int(M)]

    def evaluate(self, pop: dict, c=None, precision: str = "fp32", values: bool = True,
                 jacobian: bool = False, blocks: bool = False) -> dict:
        """One fused device pass at constants c (default c_init): per-sample values [M, N],
        Jacobian [M, K_max, N] (df/dc_k), normal-equation blocks (list of per-tree arrays:
        JtJ lower triangle packed, Jtr, 0.5*sum r^2)."""
        if self._torn:
            raise RuntimeError("InProcessCO used after teardown()")
        M, N, K_max = int(pop["M"]), int(pop["N"]), int(pop["K_max"])
        y_shared = np.asarray(pop["ym"]).ndim == 1
        hdr = build_header(pop)
        args, keep = self._inputs(pop, y_shared=y_shared)
        nt_p, nv_p, ci_p, metas_buf, _c0, xs_p, ym_p = args
        c = np.ascontiguousarray(pop["c_init"] if c is None else c, np.float64)
        vals = np.zeros((M, N), np.float64) if values else None
        jac = np.zeros((M, max(K_max, 1), N), np.float64) if jacobian else None
        Ks = np.asarray(pop["metas"], np.int64).reshape(-1, 4)[:, 3]
        nblk = int(np.sum((Ks + 1) * (Ks + 2) // 2))
        blk = np.zeros(max(nblk, 1), np.float64) if blocks else None

        def p64(a):
            return a.ctypes.data_as(_F64) if a is not None else None

        rc = self._lib.co_evaluate(
            self._handle, ctypes.byref(hdr), nt_p, nv_p, ci_p, metas_buf, p64(c), xs_p, ym_p,
            prec_code(precision), 1 if y_shared else 0,
            p64(vals), p64(jac), p64(blk))
        del keep
        if rc != CO_OK:
            raise COError(rc, "co_evaluate")
        out: dict = {}
        if values:
            out["values"] = vals
        if jacobian:
            out["jacobian"] = jac
        if blocks:
            parts, o = [], 0
            for K in Ks:
                n = int((K + 1) * (K + 2) // 2)
                parts.append(blk[o:o + n])
                o += n
            out["blocks"] = parts
        return out

    def jacobian_fd(self, pop: dict, c=None, precision: str = "fp32", eps: float = 0.0):
        """Finite-difference Jacobian [M, K_max, N] on the device (co_jacobian_fd; the
        reference FD variant's forward difference, eps <= 0: 1e-3 fp32 / 1e-7 fp64)."""
        if self._torn:
            raise RuntimeError("InProcessCO used after teardown()")
        M, N, K_max = int(pop["M"]), int(pop["N"]), int(pop["K_max"])
        y_shared = np.asarray(pop["ym"]).ndim == 1
        hdr = build_header(pop)
        args, keep = self._inputs(pop, y_shared=y_shared)
        nt_p, nv_p, ci_p, metas_buf, _c0, xs_p, ym_p = args
        c = np.ascontiguousarray(pop["c_init"] if c is None else c, np.float64)
        jac = np.zeros((M, max(K_max, 1), N), np.float64)
        rc = self._lib.co_jacobian_fd(
            self._handle, ctypes.byref(hdr), nt_p, nv_p, ci_p, metas_buf,
            c.ctypes.data_as(_F64), xs_p, ym_p, prec_code(precision), 1 if y_shared else 0,
            float(eps), jac.ctypes.data_as(_F64))
        del keep
        if rc != CO_OK:
            raise COError(rc, "co_jacobian_fd")
        return jac

    def probe_peak(self) -> tuple[float, float]:
        """Measured (fp32, fp64) FMA peak of the device in TFLOP/s."""
        a, b = ctypes.c_double(), ctypes.c_double()
        rc = self._lib.co_probe_peak(self._handle, ctypes.byref(a), ctypes.byref(b))
        if rc != CO_OK:
            raise COError(rc, "co_probe_peak")
        return a.value, b.value

    def stats(self) -> dict:
        st = CoStats()
        rc = self._lib.co_get_stats(self._handle, ctypes.byref(st))
        if rc != CO_OK:
            raise COError(rc, "co_get_stats")
        return {name: getattr(st, name) for name, _ in CoStats._fields_ if name != "reserved"}

    def last_split(self):
        s = ctypes.c_double(-1.0)
        l = ctypes.c_double(-1.0)
        rc = self._lib.co_last_split(ctypes.byref(s), ctypes.byref(l))
        if rc != 0:
            return (None, None)
        return (s.value, l.value)

    def teardown(self):
        if self._torn:
            return
        if self._handle:
            self._lib.co_teardown(self._handle)
            self._handle = ctypes.c_void_p()
        self._torn = True

    def __del__(self):
        try:
            self.teardown()
        except Exception:  # noqa: BLE001
            pass


_SINGLETONS: dict[tuple[int, str], InProcessCO] = {}
_SINGLETON_LOCK = threading.Lock()
_ATEXIT_REGISTERED = False


def _so_path(variant: str) -> Path:
    """libcusr_co_{variant}.so next to this module (aliases of libcusr_b200.so)."""
    return _HERE / f"libcusr_co_{variant}.so"


def _teardown_all() -> None:
    for co in list(_SINGLETONS.values()):
        try:
            co.teardown()
        except Exception:  # noqa: BLE001
            pass
    _SINGLETONS.clear()


def get_inproc_co(device_id: int = 0, variant: str = "ad") -> InProcessCO:
    """Process-wide InProcessCO per (device_id, variant); torn down at exit."""
    global _ATEXIT_REGISTERED
    key = (int(device_id), str(variant))
    with _SINGLETON_LOCK:
        co = _SINGLETONS.get(key)
        if co is None or co._torn:
            so = _so_path(variant)
            if not so.exists():
                raise FileNotFoundError(
                    f"{so.name} not built — run `python -m cusr_b200.build` in {_HERE.parent}")
            co = InProcessCO(device_id=device_id, lib_path=str(so), variant=variant)
            _SINGLETONS[key] = co
            if not _ATEXIT_REGISTERED:
                atexit.register(_teardown_all)
                _ATEXIT_REGISTERED = True
        return co
