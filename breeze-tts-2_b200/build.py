"""Build libbreeze_b200.so (sm_100a) in-tree with nvcc.

    python breeze-tts-2_b200/build.py [--force] [--jobs N]

Compiles every csrc/*.cu as relocatable device code for
``-gencode arch=compute_100a,code=sm_100a`` and links them, with the CUDA
runtime linked statically, into breeze_b200/libbreeze_b200.so next to the
Python package that loads it. Objects go to _build/ (git-ignored). The
library depends on nothing from PyTorch.
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
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "breeze_b200" / "libbreeze_b200.so"
BUILD = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=true", "--expt-relaxed-constexpr",
          f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), INCLUDE / "breeze_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s)]

    def compile_one(so):
        s, o = so
        cmd = [nvcc(), *ARCH, *CFLAGS, "-c", str(s), "-o", str(o)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s.name}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        for log in ex.map(compile_one, todo):
            if verbose and log:
                print(log)
    if todo or force or not OUT.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-cudart", "static",
               *map(str, objs), "-o", str(OUT)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose))
    sys.exit(0)
