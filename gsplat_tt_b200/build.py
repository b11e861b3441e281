"""Build libgs200.so (sm_100a) in-tree with nvcc.

    python -m gsplat_tt_b200.build [--force]

Steps: generate the host-logf exception table (csrc/gen_logf_table.c, run with this
host's C library), compile every csrc/*.cu for sm_100a, and link
gsplat_tt_b200/libgs200.so (static cudart, so the library only needs the driver).
display.cu and train_project.cu are compiled with -fmad=false so their float arithmetic
rounds like the reference's -ffp-contract=off CPU build and the oracle's numpy lanes; the
other units keep FMA contraction.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
GEN = os.path.join(BUILD, "gen")
LIB = os.path.join(HERE, "libgs200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
          "--expt-relaxed-constexpr", f"-I{CSRC}", f"-I{GEN}",
          f"-I{os.path.join(os.path.dirname(HERE), 'include')}"]
NO_FMA = ["-fmad=false", "-prec-div=true", "-prec-sqrt=true"]
PER_FILE = {"display.cu": NO_FMA, "train_project.cu": NO_FMA}


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def gen_logf_table(force: bool = False) -> str:
    os.makedirs(GEN, exist_ok=True)
    src = os.path.join(CSRC, "gen_logf_table.c")
    exe = os.path.join(BUILD, "gen_logf_table")
    out = os.path.join(GEN, "logf_table.inc")
    if force or _newer(exe, [src]):
        _run(["gcc", "-O2", "-o", exe, src, "-lm"])
    if force or _newer(out, [exe]):
        _run([exe, out])
    return out


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    gen_logf_table(force)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "gs200.h"))
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    jobs = []
    objs = []
    for f in sources:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-3] + ".o")
        objs.append(obj)
        deps = [src] + headers + ([os.path.join(GEN, "logf_table.inc")] if f == "display.cu" else [])
        if force or _newer(obj, deps):
            jobs.append([NVCC, *ARCH, *COMMON, *PER_FILE.get(f, []), "-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd in jobs:
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
        list(ex.map(_run, jobs))
    if force or jobs or _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
