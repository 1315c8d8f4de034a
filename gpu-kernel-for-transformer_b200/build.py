"""Compile the CUDA sources into the in-tree C-ABI library ``lib/libtfx_b200.so``.

Plain nvcc, sm_100a only (tcgen05/TMA need the arch-specific target), static
CUDA runtime, one object per translation unit compiled in parallel. The
library exports exactly the ``extern "C"`` entry points of ``include/tfx.h``
and depends on nothing torch-specific, so any host language can bind it.

    python gpu-kernel-for-transformer_b200/build.py [-v]
"""

from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PKG_DIR = pathlib.Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libtfx_b200.so"
OBJ_DIR = PKG_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-I",
    str(ROOT / "include"),
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _compile(src: pathlib.Path, verbose: bool) -> pathlib.Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    return obj


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*")) + [ROOT / "include" / "tfx.h", pathlib.Path(__file__)]
    return all(p.stat().st_mtime <= built for p in deps if p.exists())


def build(verbose: bool = False, force: bool = False) -> pathlib.Path:
    """Build (if stale) and return the path of the shared library."""
    if not force and up_to_date():
        return LIB_PATH
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
           *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv or "-v" in sys.argv))
