"""The reference's own ctypes loader binds this library unchanged.

cusr/kernel/co_inproc.py (InProcessCO, get_inproc_co) is imported from the reference checkout
(CUSR_REFERENCE, or a checkout named `reference` beside this repository) and pointed at this
repository's libcusr_co_ad.so. Without a GPU its co_init must fail the way the reference's
own library fails without a device: CO_ERR_CUDA, raised as the loader's COError with its
message. Every symbol and argument list the loader binds must resolve in this library.
Skipped where the reference is not present (the GPU box has no reference checkout).
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _reference_co_inproc():
    for cand in (os.environ.get("CUSR_REFERENCE"), str(ROOT.parent / "reference")):
        if cand and (Path(cand) / "cusr" / "kernel" / "co_inproc.py").is_file():
            path = Path(cand) / "cusr" / "kernel" / "co_inproc.py"
            spec = importlib.util.spec_from_file_location("ref_co_inproc", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
    pytest.skip("reference checkout not present")


def _lib(name: str) -> Path:
    p = ROOT / "cusr_b200" / name
    if not p.exists():
        pytest.skip(f"{name} not built")
    return p


def test_reference_structs_match_ours():
    ref = _reference_co_inproc()
    from cusr_b200 import co_inproc as ours

    for cls in ("PopHeader", "TreeMeta"):
        a, b = getattr(ref, cls), getattr(ours, cls)
        assert ctypes.sizeof(a) == ctypes.sizeof(b)
        assert [f[0] for f in a._fields_] == [f[0] for f in b._fields_]
    for code in ("CO_OK", "CO_ERR_BOUNDS", "CO_ERR_CUDA", "CO_ERR_SUM_C", "CO_ERR_SUM_NODES",
                 "CO_ERR_NULLARG", "CO_ERR_OOM"):
        assert getattr(ref, code) == getattr(ours, code)


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-device path")
def test_reference_loader_binds_library_and_reports_no_device():
    ref = _reference_co_inproc()
    lib = _lib("libcusr_co_ad.so")
    with pytest.raises(ref.COError) as ei:
        ref.InProcessCO(device_id=0, lib_path=str(lib), variant="ad")
    assert ei.value.code == ref.CO_ERR_CUDA
    assert "co_init" in str(ei.value)
    # the symbols and signatures the loader binds resolve in this library
    cdll = ctypes.CDLL(str(lib.resolve()))
    for sym in ("co_init", "co_optimize", "co_teardown", "co_last_split"):
        assert hasattr(cdll, sym), sym
    s, l = ctypes.c_double(0.0), ctypes.c_double(0.0)
    cdll.co_last_split.argtypes = [ctypes.POINTER(ctypes.c_double)] * 2
    assert cdll.co_last_split(ctypes.byref(s), ctypes.byref(l)) == 0
    cdll.co_teardown.argtypes = [ctypes.c_void_p]
    cdll.co_teardown(None)                 # NULL-safe, as the reference's


def test_fd_library_has_its_own_co_optimize():
    """libcusr_co_fd.so defines co_optimize (the FD acceptance order) and takes co_init,
    co_last_split, co_teardown and the extended symbols from libcusr_b200.so."""
    fd = ctypes.CDLL(str(_lib("libcusr_co_fd.so").resolve()))
    base = ctypes.CDLL(str(_lib("libcusr_b200.so").resolve()))

    def addr(f):
        return ctypes.cast(f, ctypes.c_void_p).value

    assert addr(fd.co_optimize) != addr(base.co_optimize)
    for sym in ("co_init", "co_teardown", "co_last_split", "co_optimize_ex"):
        assert addr(getattr(fd, sym)) == addr(getattr(base, sym)), sym
