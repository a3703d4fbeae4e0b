"""cusr_b200 — Blackwell-native (sm_100a) batched Levenberg–Marquardt constant fitting for
populations of symbolic-regression expression trees in the CuSR pop.bin bytecode.

    from cusr_b200 import get_inproc_co
    co = get_inproc_co(device_id=0)
    out = co.optimize(pop, max_iter=50)          # reference-compatible (fp32)
    out = co.optimize_ex(pop, precision="fp64")  # extended entry

The fits run in libcusr_b200.so (hand-written CUDA for sm_100a); build it with
`python -m cusr_b200.build`. There is no CPU fallback.
"""
from .co_inproc import (COError, InProcessCO, PopHeader, TreeMeta, get_inproc_co,  # noqa: F401
                        load_library)

__all__ = ["COError", "InProcessCO", "PopHeader", "TreeMeta", "get_inproc_co", "load_library"]
