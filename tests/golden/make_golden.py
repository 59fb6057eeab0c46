"""Generates the golden fixtures in this directory from the reference's own
kernels (fastgs_core/metal/*.metal compiled for the CPU into oracle/_ref by
oracle/build.py). Run where the reference tree exists:

    python oracle/build.py && python tests/golden/make_golden.py

Cases (inputs restate the reference's fixtures; outputs come from its kernels):
  tile_prep_hand   scripts/tile_prep_smoke.py:26-35 (8 hand-built keys, 4 tiles)
  raster_one       scripts/rasterize_backward_validation.py:28-45 (one splat, 16x16)
  preprocess_line8 scripts/preprocess_backward_validation.py:28-57 (8 Gaussians)
  e2e16            scripts/e2e_backward_smoke.py:31-45 (16 Gaussians, 32x32;
                   the colors_precomp path, since the reference fixture also
                   passes dc/sh and its binding then rejects the call)
  rand_sh3         seeded 300-Gaussian SH-degree-3 scene, 40x24 (partial tiles)
  config1          BASELINE config 1 (2048 Gaussians, 256x256, SH 0): SHA-256
                   of every output plus sampled values
Backward passes use the cotangent of loss = sum(out_color * w) with a seeded w.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from fastgs_core_b200 import synthetic as S  # noqa: E402
from oracle.oracle import RefKernels  # noqa: E402

FWD_KEYS = ("radii", "xys", "depths", "cov3d", "rgb", "conic_opacity", "tiles_touched", "clamped",
            "viewspace_points", "point_offsets", "point_list_keys_unsorted", "point_list_unsorted",
            "point_list_keys", "point_list", "ranges", "bucket_count", "bucket_offsets",
            "bucket_to_tile", "sampled_t", "sampled_ar", "final_t", "n_contrib", "max_contrib",
            "pixel_colors", "out_color")
BWD_KEYS = ("dmeans2d", "dcolors", "dconic_opacity", "dviewspace_raster", "dmeans3d", "ddc", "dsh",
            "dcolors_precomp", "dopacities", "dscales", "dquats", "dviewspace_points")


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def chain(ref, ins, W, H, tanx, tany, degree, seed):
    f = ref.forward(ins, W=W, H=H, tan_fovx=tanx, tan_fovy=tany, degree=degree)
    w = np.random.default_rng(seed).uniform(-1, 1, (3, W * H)).astype(np.float32)
    b = ref.backward(f, w)
    return f, b, w


def e2e16_inputs():
    n = 16
    return dict(
        background=np.zeros(3, np.float32),
        means3d=np.array([[0.1, 0.1, 1.2 + 0.01 * i] for i in range(n)], np.float32),
        colors_precomp=np.tile(np.array([[1.0, 0.6, 0.2]], np.float32), (n, 1)),
        opacities=np.full(n, 0.6, np.float32),
        cov3d_precomp=np.tile(np.array([[1.0, 0.0, 0.0, 1.0, 0.0, 1.0]], np.float32), (n, 1)),
        metric_map=np.zeros(32 * 32, np.int32),
        viewmatrix=np.eye(4, dtype=np.float32), projmatrix=np.eye(4, dtype=np.float32),
        campos=np.zeros(3, np.float32), viewspace_points=np.zeros((n, 4), np.float32))


def line8_inputs():
    m = np.array([[0.1, 0.2, 1.0], [0.2, 0.1, 1.1], [0.3, 0.0, 1.2], [0.0, 0.3, 1.3],
                  [0.1, 0.1, 1.4], [0.2, 0.2, 1.5], [0.3, 0.3, 1.6], [0.4, 0.2, 1.7]], np.float32)
    n = 8
    return dict(means3d=m, opacities=np.ones(n, np.float32), cov3d_precomp=np.ones((n, 6), np.float32),
                colors_precomp=np.ones((n, 3), np.float32), viewmatrix=np.eye(4, dtype=np.float32),
                projmatrix=np.eye(4, dtype=np.float32), campos=np.zeros(3, np.float32),
                background=np.zeros(3, np.float32), metric_map=np.zeros(256, np.int32),
                viewspace_points=np.zeros((n, 4), np.float32))


def main() -> int:
    ref = RefKernels()
    out = {}

    # tile prep, hand keys
    keys = np.array([(0 << 32) | 1, (0 << 32) | 2, (1 << 32) | 1, (1 << 32) | 2, (1 << 32) | 3,
                     (3 << 32) | 1, (3 << 32) | 2, (3 << 32) | 3], np.uint64)
    ranges = np.zeros((4, 2), np.uint32)
    bc = np.zeros(4, np.uint32)
    ref.tile_prep(8, 4, keys, ranges, bc)
    np.savez_compressed(os.path.join(HERE, "tile_prep_hand.npz"), keys=keys, ranges=ranges,
                        bucket_count=bc)
    out["tile_prep_hand"] = ranges.tolist()

    # one splat, rasterize forward + backward through the reference kernels
    W = H = 16
    a = dict(ranges=np.array([[0, 1]], np.uint32), point_list=np.array([0], np.uint32),
             bucket_offsets=np.array([1], np.uint32), means2d=np.array([[8.0, 8.0]], np.float32),
             colors=np.array([[1.0, 0.5, 0.25]], np.float32),
             conic_opacity=np.array([[1.0, 0.0, 1.0, 0.5]], np.float32),
             background=np.zeros(3, np.float32), radii=np.array([1], np.int32),
             metric_map=np.zeros(256, np.int32), bucket_to_tile=np.zeros(256, np.uint32),
             sampled_t=np.zeros(256, np.float32), sampled_ar=np.zeros(3 * 256 + 96, np.float32),
             final_t=np.zeros(256, np.float32), n_contrib=np.zeros(256, np.uint32),
             max_contrib=np.zeros(1, np.uint32), pixel_colors=np.zeros((3, 256), np.float32),
             out_color=np.zeros((3, 256), np.float32), metric_count=np.zeros(1, np.int32),
             metric_count_buf=np.zeros(1, np.int32))
    ref.render_forward(W, H, 1, 1, 0, a)
    w = np.random.default_rng(1).uniform(-1, 1, (3, 256)).astype(np.float32)
    g = dict(dL_dout=w, dmeans2d=np.zeros((1, 2), np.float32), dcolors=np.zeros((1, 3), np.float32),
             dconic=np.zeros((1, 4), np.float32), dviewspace=np.zeros((1, 4), np.float32))
    ref.render_backward(W, H, 1, 1, a, g)
    np.savez_compressed(os.path.join(HERE, "raster_one.npz"), dL_dout=w,
                        **{k: a[k] for k in ("means2d", "colors", "conic_opacity", "bucket_to_tile",
                                             "sampled_t", "final_t", "n_contrib", "max_contrib",
                                             "pixel_colors", "out_color")},
                        sampled_ar=a["sampled_ar"][:768],
                        **{k: g[k] for k in ("dmeans2d", "dcolors", "dconic", "dviewspace")})

    # preprocess line of 8 and the 16-Gaussian e2e chain (colors_precomp + cov3d_precomp)
    for name, ins, W, H in (("preprocess_line8", line8_inputs(), 16, 16), ("e2e16", e2e16_inputs(), 32, 32)):
        f, b, w = chain(ref, ins, W, H, 1.0, 1.0, 0, 2)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), cotangent=w,
                            **{"in_" + k: v for k, v in ins.items()},
                            **{"f_" + k: f[k] for k in FWD_KEYS if k in f},
                            **{"b_" + k: v for k, v in b.items()})
        out[name] = int(f["rendered"])

    # seeded SH-3 scene with partial tiles
    scene, cam = S.small_scene(11, 300, 3, 40, 24)
    ins = S.render_inputs(scene, cam, (0.2, 0.1, 0.05))
    f, b, w = chain(ref, ins, cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, 3, 3)
    np.savez_compressed(os.path.join(HERE, "rand_sh3.npz"), cotangent=w,
                        **{"f_" + k: f[k] for k in FWD_KEYS if k in f},
                        **{"b_" + k: v for k, v in b.items()})
    out["rand_sh3"] = int(f["rendered"])

    # config 1: hashes of every output plus a few hundred sampled values
    scene, cams = S.config1(0)
    cam = cams[0]
    ins = S.render_inputs(scene, cam)
    f, b, w = chain(ref, ins, cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, 0, 4)
    rng = np.random.default_rng(5)
    pix = rng.integers(0, cam.width * cam.height, 256)
    gi = rng.integers(0, scene.n, 256)
    lines = [f"rendered {f['rendered']}", f"num_buckets {f['num_buckets']}"]
    # max_contrib excluded: the reference reads unwritten threadgroup slots on partial tiles
    lines += [f"fwd {k} {sha(f[k])}" for k in FWD_KEYS if k in f and k != "max_contrib"]
    lines += [f"bwd {k} {sha(v)}" for k, v in b.items()]
    with open(os.path.join(HERE, "config1.sha256"), "w") as fh:
        fh.write("\n".join(lines) + "\n")
    np.savez_compressed(os.path.join(HERE, "config1_samples.npz"), pix=pix, gi=gi,
                        out_color=f["out_color"][:, pix], n_contrib=f["n_contrib"][pix],
                        final_t=f["final_t"][pix], tiles_touched=f["tiles_touched"][gi],
                        radii=f["radii"][gi], dmeans3d=b["dmeans3d"][gi], dscales=b["dscales"][gi],
                        dquats=b["dquats"][gi], dopacities=b["dopacities"][gi], ddc=b["ddc"][gi])
    out["config1"] = int(f["rendered"])
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
