"""Builds libmoe_b200.so in-tree with nvcc for sm_100a (cross-compiles without a GPU).

    python -m moe_swarm_b200.build [--verbose]

The library is plain CUDA C++ with a C ABI (include/moe_b200.h); it links the CUDA
runtime statically and reaches the driver's cuTensorMapEncodeTiled through
cudaGetDriverEntryPointByVersion, so it needs no libcuda at link time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmoe_b200.so"
TRACE_LIB = PKG / "libmoe_b200_trace.so"   # MOE_TRACE build: per-CTA role counters
SOURCES = ["route.cu", "wide.cu", "stream.cu", "combine.cu", "ep.cu", "capi.cu"]
HEADERS = ["ptx.cuh", "moe_internal.cuh", "launch_args.cuh", "sched.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden",
         # role timers exist only in MOE_TRACE builds; elsewhere they are unused locals
         "-diag-suppress", "177,550"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "moe_b200.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False,
          trace: bool = False) -> Path:
    lib = TRACE_LIB if trace else LIB
    if not force and not trace and not needs_build():
        return LIB
    objs = []
    build_dir = PKG / ("_build_trace" if trace else "_build")
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *FLAGS, "-I", str(ROOT / "include"), "-c", str(CSRC / src), "-o", str(obj)]
        if trace:
            cmd.append("-DMOE_TRACE")
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build libmoe_b200_trace.so with MOE_TRACE")
    a = ap.parse_args(argv)
    print(build(verbose=a.verbose, force=a.force or a.ptxas_verbose, ptxas_verbose=a.ptxas_verbose,
                trace=a.trace))


if __name__ == "__main__":
    main(sys.argv[1:])
