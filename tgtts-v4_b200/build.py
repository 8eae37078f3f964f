"""Builds libtgcuda.so, the kernels and runtime behind include/tgcuda.h, for sm_100a only.

Each .cu under csrc/ is compiled by nvcc with -gencode arch=compute_100a,code=sm_100a into an
object, and the objects are linked into lib/libtgcuda.so (CUDA runtime linked statically). A
source is recompiled when it or a header is newer than its object. Nothing here needs a GPU.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "build"
LIB = PKG / "lib" / "libtgcuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall,-Wextra", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libtgcuda.so")
    return found


def _headers_mtime() -> float:
    heads = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in heads), default=0.0)


def _compile(src: Path, newest_header: float, verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if res.stderr and (verbose or "warning" in res.stderr):
        print(res.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    """Compiles what changed and links lib/libtgcuda.so; returns its path."""
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    newest = _headers_mtime()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda s: _compile(s, newest, verbose), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"linking libtgcuda.so failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    import sys

    print(build(verbose="-v" in sys.argv))
