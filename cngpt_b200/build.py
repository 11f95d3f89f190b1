"""Build libcngpt_cuda.so in-tree (sm_100a only).

    python -m cngpt_b200.build          # or: python cngpt_b200/build.py

Every .cu under csrc/ is compiled by nvcc for compute_100a/sm_100a with
-lineinfo into _build/, then linked into cngpt_b200/libcngpt_cuda.so with the
static CUDA runtime; NCCL is opened at run time when data parallelism starts. Rebuilds only what changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "cngpt_cuda"
LIB = PKG / "libcngpt_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "-diag-suppress", "20044", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _host_cc() -> list[str]:
    # the image's default CC lacks libgomp; nvcc only needs a plain g++
    gxx = "/usr/bin/g++"
    return ["-ccbin", gxx] if Path(gxx).exists() else []


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").rglob("*.h"))
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if _stale(obj, src):
        cmd = [nvcc(), *_host_cc(), *ARCH, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-I", str(CSRC),
               "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *_host_cc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs),
               "-ldl", "-Xlinker", "-soname=libcngpt_cuda.so", "-Xlinker", "-Bsymbolic"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
