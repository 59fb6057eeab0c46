"""Builds libfastgs_b200.so (all CUDA kernels + the C ABI) for sm_100a.

nvcc cross-compiles without a GPU. Objects go to fastgs_core_b200/_build/,
the library next to the package (fastgs_core_b200/libfastgs_b200.so), so the
built file travels with the repository snapshot.

Flags: -gencode arch=compute_100a,code=sm_100a -lineinfo -O3; -fmad=false
(no multiply-add contraction) for the files whose kernels must reproduce the
CPU checker bit for bit (fused operations appear there only where the source
writes fmaf). raster_bwd.cu and train.cu may contract: their gradients are
compared within tolerance, and the one exact decision in raster_bwd.cu (the
alpha test shared with the forward pass) uses explicitly rounded intrinsics.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfastgs_b200.so")
SOURCES = ["preprocess.cu", "binning.cu", "raster.cu", "raster_bwd.cu", "train.cu", "densify.cu"]
# files whose kernels may contract multiply-adds (their exact decisions use
# explicitly rounded intrinsics)
FMAD_OK = {"raster_bwd.cu", "train.cu"}
HEADERS = ["fgs_common.cuh", "tile_walk.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _newest_dep() -> float:
    paths = [os.path.join(HERE, h) for h in HEADERS]
    paths.append(os.path.join(PKG, os.pardir, "include", "fastgs_b200.h"))
    return max(os.path.getmtime(p) for p in paths if os.path.exists(p))


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    srcp = os.path.join(HERE, src)
    if (os.path.exists(obj) and os.path.getmtime(obj) > os.path.getmtime(srcp)
            and os.path.getmtime(obj) > _newest_dep() and not verbose_ptxas):
        return obj
    flags = [f for f in FLAGS if not (src in FMAD_OK and f == "-fmad=false")]
    cmd = [NVCC, *flags, "-c", srcp, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas or r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(HERE, s))]
    if force:
        for s in srcs:
            o = os.path.join(BUILD, os.path.splitext(s)[0] + ".o")
            if os.path.exists(o):
                os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB,
               "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
