"""Builds libflowmoe.so in-tree (openflowlm-next_b200/flowmoe/libflowmoe.so) for sm_100a.

    python openflowlm-next_b200/build.py [--force] [--verbose]

One nvcc invocation over csrc/*.cu, -gencode arch=compute_100a,code=sm_100a. The library is a plain C
ABI (include/flowmoe.h) with no torch dependency; flowmoe/_lib.py loads it with ctypes.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "flowmoe" / "libflowmoe.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or Path(c).exists()):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "flowmoe.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include"), "-I", str(CSRC),
           "-o", str(OUT) + ".tmp", *map(str, sources()), "-lcuda",
           "-Xlinker", "-rpath=" + str(Path(nvcc()).resolve().parent.parent / "lib64")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libflowmoe.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
