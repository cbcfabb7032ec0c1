"""Build librembed_gpu.so (sm_100a) in-tree with nvcc.

    python -m rembed_b200.build          # incremental
    python -m rembed_b200.build --force  # rebuild everything

Each .cu compiles to an object under rembed_b200/_build/ in parallel, then
links into rembed_b200/librembed_gpu.so (static CUDA runtime, so the
library needs only the driver at run time).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "librembed_gpu.so"
INCLUDE = PKG.parent / "include"
SOURCES = ["gemm.cu", "gemm_kind_bf16.cu", "gemm_kind_s8.cu", "gemm_kind_f16.cu", "gemm_kind_w8.cu",
           "gemm_kind_tf32x3.cu", "kernels.cu", "attention_tc.cu", "runtime.cu", "noalloc.cu",
           "kernel_abi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    jobs = []
    for s in SOURCES:
        src, obj = CSRC / s, BUILD / (Path(s).stem + ".o")
        if force or _stale(obj, src):
            jobs.append([cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose or res.returncode:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    objs = [str(BUILD / (Path(s).stem + ".o")) for s in SOURCES]
    if force or jobs or not LIB.exists():
        res = subprocess.run([cc, *ARCH, "-shared", "-o", str(LIB), *objs], capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of librembed_gpu.so failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
