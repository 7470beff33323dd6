"""Builds ``lib/libh3b.so`` (the C-ABI library) from ``csrc/*.cu`` with nvcc for sm_100a.

Usage: ``python fasth3-gb300_b200/build.py [-j N] [--force]``. Objects are rebuilt only when a source or header is
newer than them. The quantizer translation unit is compiled with ``--use_fast_math`` (the reference extension's flag,
fastvideo/models/dits/h3fast/__init__.py:42) so its arithmetic matches the reference bit for bit; the others are not.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "lib" / "libh3b.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC),
          "--expt-relaxed-constexpr"]
FAST_MATH = {"quant.cu", "vsa_prologue.cu", "gate_quant.cu"}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def compile_one(src: Path, force: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if force or _stale(obj, src):
        flags = list(COMMON)
        if src.name in FAST_MATH:
            flags.append("--use_fast_math")
        cmd = [nvcc(), *ARCH, *flags, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(jobs: int = 8, force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force), sources))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    try:
        build(a.j, a.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
