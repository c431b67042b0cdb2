"""Build libdspine_b200.so (all CUDA sources under csrc/) for sm_100a, in-tree.

    python -m dspine_b200.build          # or dspine_b200.build.build()

The shared library carries the C ABI declared in include/dspine_b200.h and is loaded with
ctypes by dspine_b200._lib.  Objects are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "_lib"
LIB = OUT_DIR / "libdspine_b200.so"
OBJ_DIR = ROOT / "_build" / "obj"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include")]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build dspine_b200")
    return path


def _host_compiler_args():
    # some images export CC/CXX pointing at a wrapper; nvcc picks its host compiler from PATH
    gxx = "/usr/bin/g++"
    return ["-ccbin", gxx] if Path(gxx).exists() else []


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def build(verbose: bool = False, ptxas_info: bool = False, checked: bool = False,
          profile: bool = False) -> Path:
    """Compile every csrc/*.cu and link the shared library.  ``checked`` builds the index-
    checking variant (-DDSV_CHECKS) into _build/checked/, ``profile`` the phase-timing variant
    (-DDSV_PROFILE) into _build/profile/, instead of the product library."""
    variant = "checked" if checked else ("profile" if profile else None)
    out_dir = (ROOT / "_build" / variant) if variant else OUT_DIR
    obj_dir = OBJ_DIR.parent / (f"obj_{variant}" if variant else "obj")
    lib = out_dir / LIB.name
    out_dir.mkdir(parents=True, exist_ok=True)
    obj_dir.mkdir(parents=True, exist_ok=True)
    extra = (["-DDSV_CHECKS"] if checked else []) + (["-DDSV_PROFILE"] if profile else [])
    cc = nvcc()
    hdr_mtime = max((p.stat().st_mtime for p in headers()), default=0)
    objs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
            continue
        cmd = [cc, *ARCH, *FLAGS, *extra, *_host_compiler_args(), "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    newest = max(o.stat().st_mtime for o in objs)
    if not lib.exists() or lib.stat().st_mtime < newest:
        cmd = [cc, *ARCH, *_host_compiler_args(), "-shared", "-o", str(lib), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return lib


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="-v" in sys.argv, checked="--checked" in sys.argv,
                profile="--profile" in sys.argv))
