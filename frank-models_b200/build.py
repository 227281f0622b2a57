"""Build ``libfrankmoe.so`` in-tree with nvcc for sm_100a.

Usage: ``python frank-models_b200/build.py [--force]``.  The library lands in
``frank-models_b200/frank_b200/libfrankmoe.so`` next to the Python module
that loads it, so it travels with the source tree.  Rebuilds only when a
source or header is newer than the library (or with ``--force``).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
OUT = PKG_ROOT / "frank_b200" / "libfrankmoe.so"
BUILD_DIR = PKG_ROOT / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return OUT
    BUILD_DIR.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = OUT.with_suffix(".so.tmp")
    subprocess.run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
