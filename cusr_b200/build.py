"""Build libcusr_b200.so (sm_100a) in-tree.

    python -m cusr_b200.build            # incremental
    python -m cusr_b200.build --force    # rebuild everything

The library is also exposed under the file name the CuSR ctypes loader looks for
(libcusr_co_ad.so), and libcusr_co_fd.so is built beside it (the FD variant's acceptance
order, over this library), so the reference's `co_inproc.InProcessCO` binds either unchanged.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ = HERE / "_build"
LIB = HERE / "libcusr_b200.so"
ALIASES = ("libcusr_co_ad.so",)
# the FD variant's name: its own small library (co_optimize with the FD acceptance order) over
# libcusr_b200.so
FD_LIB = HERE / "libcusr_co_fd.so"
FD_SOURCE = "fd_variant.cpp"
# command-line front end with the reference binary's interface, and the names the reference's
# subprocess callers use for it
CLI = HERE / "batch_lm_b200"
CLI_SOURCE = "batch_lm_cli.cpp"
CLI_ALIASES = ("batch_lm", "batch_lm_ad")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-O3", f"-I{INCLUDE}"]
SOURCES = ["eval_f32.cu", "eval_f32_fast.cu", "eval_f64.cu", "engine.cu", "pack.cpp",
           "debug_api.cpp", "noalloc.cu", "shard_comm.cpp"]
# the reference kernel's numerics (cusr/kernel/Makefile:9) for CoOptions.math = CO_MATH_FAST
FILE_FLAGS = {"eval_f32_fast.cu": ["--use_fast_math"]}


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, defines: tuple = (), obj_dir: Path = None,
          lib: Path = None) -> Path:
    """Compile every source for sm_100a and link the library (incremental)."""
    nvcc = _nvcc()
    OBJ = obj_dir or globals()["OBJ"]
    LIB = lib or globals()["LIB"]
    OBJ.mkdir(parents=True, exist_ok=True)
    flags = NVCC_FLAGS + [f"-D{d}" for d in defines]
    hdrs = _headers()
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = OBJ / (s.stem + ".o")
        if force or _stale(o, [s, *hdrs, Path(__file__)]):
            jobs.append([nvcc, *flags, *FILE_FLAGS.get(src, []), "-c", str(s), "-o", str(o)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    objs = [OBJ / (Path(s).stem + ".o") for s in SOURCES]
    if force or jobs or _stale(LIB, objs):
        run([nvcc, *ARCH, "-shared", "-Xlinker", f"-soname={LIB.name}", "-o", str(LIB),
             *map(str, objs), "-lcudart", "-ldl"])
    if lib is not None:
        return LIB
    fd_src = CSRC / FD_SOURCE
    if FD_LIB.is_symlink():
        FD_LIB.unlink()
    if force or _stale(FD_LIB, [fd_src, LIB, *hdrs]):
        run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-I{INCLUDE}", str(fd_src), "-o",
             str(FD_LIB), f"-L{HERE}", f"-l:{LIB.name}", "-Wl,-rpath,$ORIGIN"])
    cli_src = CSRC / CLI_SOURCE
    if force or _stale(CLI, [cli_src, LIB, *hdrs]):
        run(["g++", "-O2", "-std=c++17", f"-I{INCLUDE}", str(cli_src), "-o", str(CLI),
             f"-L{HERE}", f"-l:{LIB.name}", "-Wl,-rpath,$ORIGIN"])
    for names, target in ((ALIASES, LIB.name), (CLI_ALIASES, CLI.name)):
        for alias in names:
            a = HERE / alias
            if a.is_symlink() or a.exists():
                if a.is_symlink() and os.readlink(a) == target:
                    continue
                a.unlink()
            a.symlink_to(target)
    return LIB


def ptxas_report() -> str:
    """Markdown table of every kernel's registers, stack frame and spills (ptxas -v) for the
    CUDA sources, compiled as the library build compiles them."""
    import re
    import tempfile

    nvcc = _nvcc()
    rows = []
    with tempfile.TemporaryDirectory() as tmp:
        for src in [s for s in SOURCES if s.endswith(".cu")]:
            cmd = [nvcc, *NVCC_FLAGS, *FILE_FLAGS.get(src, []), "-Xptxas", "-v", "-c",
                   str(CSRC / src), "-o", str(Path(tmp) / "x.o")]
            err = subprocess.run(cmd, capture_output=True, text=True).stderr.splitlines()
            name, frame = None, None
            for i, line in enumerate(err):
                m = re.search(r"Function properties for (\S+)", line)
                if m:
                    name = m.group(1)
                    frame = err[i + 1] if i + 1 < len(err) else ""
                    continue
                m = re.search(r"Used (\d+) registers", line)
                if m and name and name.startswith("_Z"):
                    st = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, "
                                   r"(\d+) bytes spill loads", frame or "")
                    demangled = subprocess.run(["c++filt", name], capture_output=True,
                                               text=True).stdout.strip().replace("cusr::", "")
                    if st:
                        rows.append(f"| {src} | `{demangled}` | {m.group(1)} | {st.group(1)} | "
                                    f"{st.group(2)}/{st.group(3)} |")
                    name = None
    head = ["| file | kernel | registers | stack B | spill st/ld B |", "|---|---|---|---|---|"]
    return "\n".join(head + rows)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--define", action="append", default=[],
                    help="extra preprocessor define of a variant build (e.g. CUSR_IEEE_F32: the "
                         "fp32 interpreter with the accurate library transcendentals instead "
                         "of the SFU arithmetic); needs --lib")
    ap.add_argument("--ptxas-report", action="store_true",
                    help="print every kernel's registers / stack / spills (ptxas -v) and exit")
    ap.add_argument("--lib", default=None,
                    help="output path of a variant library (objects beside it in _build/); "
                         "the in-tree library and its aliases are left as they are")
    a = ap.parse_args()
    if a.ptxas_report:
        print(ptxas_report())
        return
    if a.define and not a.lib:
        ap.error("--define builds a variant: give --lib")
    lib = Path(a.lib).resolve() if a.lib else None
    print(build(force=a.force, verbose=a.verbose, defines=tuple(a.define),
                obj_dir=lib.parent / "_build" if lib else None, lib=lib))


if __name__ == "__main__":
    main()
