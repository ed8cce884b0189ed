"""Builds libqmm.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m machinelearning_b200.build        # incremental
    python -m machinelearning_b200.build --force

The library is written next to this file so that it travels with the source
tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqmm.so")
BUILD_DIR = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O2",
    # IEEE division / square root and no flush-to-zero: the quantisers must be
    # bit-identical to the reference's CPU arithmetic.
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-fmad=true",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "qmm.h"))
    return hs


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    cmds = []
    hdrs = headers()
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            cmds.append(cmd)
    # translation units compile independently: run them side by side
    procs = [subprocess.Popen(c) for c in cmds]
    failed = [c for c, p in zip(cmds, procs) if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    if force or _stale(LIB, objs):
        # static runtime: the library does not depend on whichever libcudart.so
        # the process happens to resolve first (torch ships its own)
        cmd = [nvcc(), *ARCH, "-shared", "--cudart", "static", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
