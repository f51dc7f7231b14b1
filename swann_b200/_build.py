"""Build recipe for the CUDA library (in-tree, sm_100a).

``python -m swann_b200._build`` compiles ``csrc/*.cu`` into
``swann_b200/libswann_b200.so`` with nvcc, statically linking the CUDA runtime
so the library depends on nothing but the driver.  The built ``.so`` is
git-ignored and travels with the working tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libswann_b200.so"
SOURCES = ["search.cu", "build.cu", "sweep_mma.cu", "prune_tc.cu", "select.cu", "offline.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# The search's distance sums must round every multiply and add on its own (the
# reference builds with -fmad=false too); ptxas would otherwise fuse the packed
# f32x2 multiply-adds of the row sums, explicit rounding modifiers or not.
PER_FILE = {"search.cu": ["-fmad=false"]}


def _sources():
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def _deps():
    return _sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        [HERE.parent / "include" / "swann_b200.h", Path(__file__).resolve()]


def up_to_date() -> bool:
    return LIB.exists() and all(LIB.stat().st_mtime >= p.stat().st_mtime for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    objs = []
    build_dir = HERE / "_build"
    build_dir.mkdir(exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                    "--expt-relaxed-constexpr", "-I", str(HERE.parent / "include")]
    procs = []
    for src in _sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc] + flags + PER_FILE.get(src.name, []) + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append(subprocess.Popen(cmd))
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("nvcc failed building swann_b200")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
