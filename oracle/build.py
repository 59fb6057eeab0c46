"""Build recipe for the CPU checkers (test infrastructure, not the product).

* ``liboracle.so``       - fgs_oracle.c with the exp/log the CUDA kernels use
                           (bit-identical integer outputs and image vs the GPU)
* ``liboracle_libm.so``  - the same source with libm expf/logf, pinned
                           bit-for-bit against the reference's kernels
* ``_ref/libfgs_ref.so`` - the reference's own Metal kernels compiled as C++
                           through ref_shim/metal_stdlib, straight from the
                           read-only reference tree; only built where that tree
                           exists (the built .so travels with the repo
                           snapshot, the reference tree does not).

Run: ``python oracle/build.py [--reference-dir DIR]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def default_reference_dir() -> str:
    """The reference checkout: $FGS_REFERENCE_DIR, else a directory named
    ``reference`` beside this repository's root."""
    env = os.environ.get("FGS_REFERENCE_DIR")
    if env:
        return env
    return os.path.normpath(os.path.join(HERE, os.pardir, os.pardir, "reference"))

CFLAGS = ["-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-std=c11"]


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def _stale(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build_oracle(force: bool = False) -> None:
    src = os.path.join(HERE, "fgs_oracle.c")
    for name, extra in (("liboracle.so", []), ("liboracle_libm.so", ["-DFGS_ORACLE_LIBM"])):
        out = os.path.join(HERE, name)
        if force or _stale(out, [src]):
            _run(["gcc", *CFLAGS, *extra, src, "-o", out, "-lm"])


def build_ref(reference_dir: str | None = None, force: bool = False) -> bool:
    reference_dir = reference_dir or default_reference_dir()
    metal_dir = os.path.join(reference_dir, "fastgs_core", "metal")
    if not os.path.isdir(metal_dir):
        return False
    os.makedirs(os.path.join(HERE, "_ref"), exist_ok=True)
    out = os.path.join(HERE, "_ref", "libfgs_ref.so")
    srcs = [os.path.join(HERE, "ref_kernels.cpp"), os.path.join(HERE, "ref_shim", "metal_stdlib")]
    srcs += [os.path.join(metal_dir, f) for f in os.listdir(metal_dir) if f.endswith(".metal")]
    if force or _stale(out, srcs):
        _run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-Wno-attributes",
              "-I" + os.path.join(HERE, "ref_shim"), f"-DFGS_REF_DIR={metal_dir}",
              os.path.join(HERE, "ref_kernels.cpp"), "-o", out, "-lpthread"])
    return True


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=None,
                    help="reference checkout (default: $FGS_REFERENCE_DIR or ../reference)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build_oracle(a.force)
    ok = build_ref(a.reference_dir, a.force)
    print("oracle built; reference kernels", "built" if ok else "skipped (no reference tree)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
