"""Build libppocr_cuda.so in-tree: every CUDA source for sm_100a only.

    python ppocr-native_b200/build.py [--verbose-ptxas] [--force]

Objects go to ppocr-native_b200/_build/, the library to
ppocr-native_b200/libppocr_cuda.so (next to this file, where the ctypes
binding looks for it). nvcc links the CUDA runtime statically, so the
library needs only the driver at run time.
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
BUILD = HERE / "_build"
LIB = HERE / "libppocr_cuda.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# IEEE division and square root, no flush-to-zero: the kernels reproduce the
# reference's f32 arithmetic; every contraction is written out explicitly.
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off",
          "-ftz=false", "-prec-div=true", "-prec-sqrt=true", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.hpp")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    me = Path(__file__).stat().st_mtime
    objs = []
    todo = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        stale = (not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header, me))
        if force or stale:
            cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose and src.suffix == ".cu":
                cmd += ["-Xptxas", "-v"]
            todo.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for cmd, r in ex.map(run, todo):
            if r.returncode != 0 or (ptxas_verbose and r.stderr):
                sys.stderr.write(r.stderr)
            if r.returncode != 0:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed on {failed}")
    if force or todo or not LIB.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-Xcompiler", "-fPIC"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas_verbose=args.verbose_ptxas))
