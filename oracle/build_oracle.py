"""Build recipe for the test oracle (TEST INFRASTRUCTURE, not product code).

Two artefacts, both git-ignored (``*.so``) and both carried to the GPU box with
the working tree:

* ``oracle/liboracle.so`` -- the C restatement in ``swann_oracle.c``.
* ``oracle/_ref/swann_ref_ls*.so`` -- the reference's own search kernels
  (``swann/csrc/local_search.cu`` of geniussyn/SWANN), compiled unmodified for
  sm_100a.  The source is taken from the reference project named by the
  ``SWANN_REFERENCE`` environment variable (its root directory), else from the
  reference package installed under ``baseline/_ref`` (``baseline/install.sh``).
  It is a torch extension with the reference's pybind entry points; tests and
  the bench's baseline legs load it only as a checker or baseline.  The
  reference JIT-compiles the same file with ``-O3 -lineinfo -fmad=false``
  (swann/_engine.py:42-63); the flags are kept.

Usage:  python oracle/build_oracle.py [--ref]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_NAME = "swann_ref_ls"
INSTALLED_REF = HERE.parent / "baseline" / "_ref"


def reference_source() -> Path | None:
    """swann/csrc/local_search.cu of the reference: under $SWANN_REFERENCE when
    set, else in the installed copy under baseline/_ref; None when neither
    exists."""
    roots = []
    if os.environ.get("SWANN_REFERENCE"):
        roots.append(Path(os.environ["SWANN_REFERENCE"]))
    roots.append(INSTALLED_REF)
    for r in roots:
        src = r / "swann" / "csrc" / "local_search.cu"
        if src.exists():
            return src
    return None


def _newer(out: Path, *srcs: Path) -> bool:
    return out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs)


def build_oracle(force: bool = False) -> Path:
    src = HERE / "swann_oracle.c"
    if not force and _newer(ORACLE_SO, src):
        return ORACLE_SO
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-builtin-powf", "-fopenmp",
           "-o", str(ORACLE_SO), str(src), "-lm"]
    subprocess.run(cmd, check=True)
    return ORACLE_SO


def ref_so_path() -> Path:
    return REF_DIR / f"{REF_NAME}.so"


def build_ref(force: bool = False) -> Path | None:
    """Compile the reference's kernel file for sm_100a (only where it exists)."""
    src = reference_source()
    if src is None:
        return ref_so_path() if ref_so_path().exists() else None
    out = ref_so_path()
    if not force and _newer(out, src):
        return out
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths

    REF_DIR.mkdir(exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = []
    for p in include_paths(device_type="cuda") if "device_type" in include_paths.__code__.co_varnames \
            else include_paths(cuda=True):
        incs += ["-I", p]
    incs += ["-I", sysconfig.get_paths()["include"]]
    libs = []
    for p in library_paths(device_type="cuda") if "device_type" in library_paths.__code__.co_varnames \
            else library_paths(cuda=True):
        libs += ["-L", p]
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, str(src), "-o", str(out), "-shared", "-Xcompiler", "-fPIC",
           "-std=c++17", "-O3", "-lineinfo", "-fmad=false", "--expt-relaxed-constexpr",
           "-gencode", "arch=compute_100a,code=sm_100a",
           f"-DTORCH_EXTENSION_NAME={REF_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-Xcudafe", "--diag_suppress=20012", "-w"] + incs + libs + \
          ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(build_oracle(force=True))
    if "--ref" in sys.argv:
        print(build_ref(force=True))
