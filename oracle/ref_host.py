"""ctypes binding of oracle/_ref/libref_host.so — the reference's own host-compiled
interpreters (cusr/kernel/ad_interp.cuh, revad_interp.cuh). TEST INFRASTRUCTURE ONLY."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libref_host.so"

_I32 = ctypes.POINTER(ctypes.c_int32)
_F32 = ctypes.POINTER(ctypes.c_float)


def available() -> bool:
    return LIB.exists()


class RefHost:
    """fp32 value / reverse gradient / forward tangents of one tree at one sample, computed
    by the reference implementation."""

    def __init__(self):
        self.lib = ctypes.CDLL(str(LIB))
        self.lib.ref_value.restype = ctypes.c_float
        self.lib.ref_value.argtypes = [_I32, _F32, ctypes.c_int, _I32, _F32, _F32]
        self.lib.ref_vjp.restype = None
        self.lib.ref_vjp.argtypes = [_I32, _F32, ctypes.c_int, _I32, _F32, _F32, ctypes.c_int, _F32]
        self.lib.ref_jvp.restype = None
        self.lib.ref_jvp.argtypes = [_I32, _F32, ctypes.c_int, _I32, _F32, _F32, ctypes.c_int,
                                     ctypes.c_int, _F32, _F32]
        ms, mk, mn = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self.lib.ref_limits(ctypes.byref(ms), ctypes.byref(mk), ctypes.byref(mn))
        self.max_stack, self.max_k, self.max_nodes = ms.value, mk.value, mn.value

    @staticmethod
    def _p(a, dt, ct):
        a = np.ascontiguousarray(a, dt)
        return a, a.ctypes.data_as(ctypes.POINTER(ct))

    def value_and_grad(self, nt, nv, ci, x, c):
        K = len(c)
        nt_a, nt_p = self._p(nt, np.int32, ctypes.c_int32)
        nv_a, nv_p = self._p(nv, np.float32, ctypes.c_float)
        ci_a, ci_p = self._p(ci, np.int32, ctypes.c_int32)
        x_a, x_p = self._p(x, np.float32, ctypes.c_float)
        c_a, c_p = self._p(c if K else [0.0], np.float32, ctypes.c_float)
        g = np.zeros(max(K, 1), np.float32)
        v = self.lib.ref_value(nt_p, nv_p, len(nt_a), ci_p, x_p, c_p)
        if K:
            self.lib.ref_vjp(nt_p, nv_p, len(nt_a), ci_p, x_p, c_p, K, g.ctypes.data_as(_F32))
        return float(v), g[:K]
