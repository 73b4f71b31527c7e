"""Build libebx.so (all CUDA sources in this directory) for sm_100a, in tree.

Output: mlbricks_b200/_lib/libebx.so.  Objects go to mlbricks_b200/_lib/obj/.
Each translation unit is compiled in parallel with nvcc; the shared library
links the CUDA runtime statically so it carries no dependency on the toolkit
install of the machine that loads it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
LIB_DIR = PKG / "_lib"
OBJ_DIR = LIB_DIR / "obj"
LIB = LIB_DIR / "libebx.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(HERE)]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return path


def sources() -> list[Path]:
    return sorted(HERE.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(HERE.glob("*.cuh")) + list(HERE.glob("*.h")) + [INCLUDE / "ebx.h"]
    newest = max(p.stat().st_mtime for p in deps if p.exists())
    return obj.stat().st_mtime < newest


def compile_one(src: Path, verbose: bool = False) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if not _stale(obj, src):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stdout.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    if force:
        for o in OBJ_DIR.glob("*.o"):
            o.unlink()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    if LIB.exists() and not force and all(o.stat().st_mtime <= LIB.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
