"""Builds libmidman_gpu.so for sm_100a from csrc/ (nvcc, in-tree).

Usage: python midman-ai_b200/build.py [--force] [--jobs N]

Objects go to midman-ai_b200/_build/, the shared library to
midman-ai_b200/lib/libmidman_gpu.so. Sources are rebuilt when they, or any
header in csrc/ or include/, are newer than their object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libmidman_gpu.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3", "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def _newest_header() -> float:
    newest = 0.0
    for d in (CSRC, INCLUDE):
        for p in d.glob("*.h*"):
            newest = max(newest, p.stat().st_mtime)
        for p in d.glob("*.cuh"):
            newest = max(newest, p.stat().st_mtime)
    return newest


def _compile(src: Path, force: bool, hdr_time: float) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *NVCC_FLAGS, "-x", "cu", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    hdr_time = _newest_header()
    jobs = jobs or min(8, os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr_time), sources))
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objs),
               "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"linked {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=True))
    sys.exit(0)
