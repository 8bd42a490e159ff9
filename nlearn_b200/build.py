"""Build the sm_100a kernel library ``libnl_ops.so`` in-tree with nvcc.

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (in parallel,
skipped when up to date) and linked into ``nlearn_b200/libnl_ops.so`` with the
static CUDA runtime, so the library depends only on the driver at run time.

    python -m nlearn_b200.build          # or __graft_entry__.build()
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT = PKG / "libnl_ops.so"
BUILD_DIR = PKG.parent / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build the sm_100a kernel library")


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(nvcc: str, src: Path, obj: Path, dep_mtime: float, verbose: bool) -> str:
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, dep_mtime):
        return f"up to date: {src.name}"
    cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return f"compiled: {src.name}" + (f"\n{r.stderr}" if verbose and r.stderr else "")


def build(verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    dep = _deps_mtime()
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for msg in ex.map(lambda so: _compile(nvcc, so[0], so[1], dep, verbose), zip(srcs, objs)):
            if verbose:
                print(msg)
    newest = max(o.stat().st_mtime for o in objs)
    if not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(OUT), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
