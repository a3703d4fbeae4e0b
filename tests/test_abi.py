"""The C-ABI library loads, exports every symbol include/*.h declares, and its structures
match the ctypes mirrors — all without a GPU (no compute calls)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from cusr_b200 import co_inproc

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions(path: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", path.read_text(), flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(",
                      text, flags=re.M)


def test_headers_declare_entry_points():
    names = {n for h in HEADERS for n in declared_functions(h)}
    for n in ("co_init", "co_optimize", "co_last_split", "co_teardown", "co_optimize_ex",
              "co_get_stats", "co_evaluate", "co_load", "co_fit_loaded"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(co_inproc.default_lib_path()))
    for h in HEADERS:
        for name in declared_functions(h):
            assert hasattr(lib, name), f"{name} declared in {h.name} but not exported"


def test_ctypes_mirrors_bind_all_symbols():
    lib = co_inproc.load_library()
    assert set(co_inproc.SIGNATURES) <= {n for h in HEADERS for n in declared_functions(h)}
    assert lib.co_strerror(0) == b"ok"


def test_reference_loader_names():
    """The AD variant's name is the engine library itself; the FD variant's is a library of
    its own (its co_optimize has the FD acceptance order) linked against the engine."""
    p = co_inproc._HERE / "libcusr_co_ad.so"
    assert p.exists() and p.resolve() == co_inproc.default_lib_path().resolve()
    fd = co_inproc._HERE / "libcusr_co_fd.so"
    assert fd.exists() and not fd.is_symlink()


@pytest.mark.parametrize("struct,cname", [
    (co_inproc.PopHeader, "PopHeader"), (co_inproc.TreeMeta, "TreeMeta"),
    (co_inproc.CoOptions, "CoOptions"), (co_inproc.CoStats, "CoStats")])
def test_struct_sizes_match_c(struct, cname, tmp_path):
    src = tmp_path / "s.c"
    src.write_text(f'#include "cusr_co.h"\n#include <stdio.h>\n'
                   f'int main(void){{printf("%zu", sizeof({cname}));return 0;}}\n')
    exe = tmp_path / "s"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    size = int(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert size == ctypes.sizeof(struct)


def test_default_options_are_reference_defaults():
    lib = co_inproc.load_library()
    opt = co_inproc.CoOptions()
    lib.co_default_options(ctypes.byref(opt))
    assert opt.struct_size == ctypes.sizeof(co_inproc.CoOptions)
    assert opt.precision == 0 and opt.max_iter == 50
    assert opt.lambda0 == pytest.approx(1e-3) and opt.xtol == pytest.approx(1e-6)


def test_null_arguments_rejected_before_device_work():
    lib = co_inproc.load_library()
    hdr = co_inproc.PopHeader()
    z = np.zeros(4, np.float32)
    zi = np.zeros(4, np.int32)
    F = ctypes.POINTER(ctypes.c_float)
    I = ctypes.POINTER(ctypes.c_int32)
    rc = lib.co_optimize(None, ctypes.byref(hdr), zi.ctypes.data_as(I), z.ctypes.data_as(F),
                         zi.ctypes.data_as(I), None, z.ctypes.data_as(F), z.ctypes.data_as(F),
                         z.ctypes.data_as(F), 5, z.ctypes.data_as(F), zi.ctypes.data_as(I),
                         None, None)
    assert rc == co_inproc.CO_ERR_NULLARG
    assert lib.co_get_stats(None, None) == co_inproc.CO_ERR_NULLARG
    lib.co_teardown(None)   # NULL-safe
    out = ctypes.c_void_p()
    assert lib.co_init(0, None) == co_inproc.CO_ERR_NULLARG


def test_last_split_always_reports():
    lib = co_inproc.load_library()
    a, b = ctypes.c_double(), ctypes.c_double()
    assert lib.co_last_split(ctypes.byref(a), ctypes.byref(b)) == 0
