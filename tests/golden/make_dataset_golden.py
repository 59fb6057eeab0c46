"""Generates tests/golden/dataset_ref.npz by running the reference's own scanner
dataset loader (test infrastructure; run where the reference tree exists):

    python tests/golden/make_dataset_golden.py [--reference-dir DIR]

The reference reads a scanner capture (frame_*.jpg + frame_*.json pairs and a
points.ply) in scripts/train_scanner_fixed.py:237-498 (collect_scanner_frames,
compute_normalization, build_camera_from_scanner_json, load_target_image,
prepare_dataset) and seeds the model in init_model (:601-628). Its module
imports mlx, cv2 and plyfile, none of which is installable here: this script
puts stand-ins for them in sys.modules (NumPy arrays behind the mlx names the
loader calls; a binary-little-endian vertex reader behind plyfile.PlyData; an
empty cv2, which the loader never calls) and imports the unmodified script.

The capture itself is made here, seeded, and stored in the fixture as file
bytes, so the test writes the same files and runs this repository's loader on
them. Cases:
  plain   4 frames at 64x48 rendered at 32x24 (bilinear resize), rotated poses,
          coloured points, no subsampling, no extra points
  jitter  frame_step 2 from index 1, max_points below the point count
          (rng.choice), surface-jitter extra points
  bbox    bbox extra points, points without colours (the 0.5 default)
"""
from __future__ import annotations

import argparse
import importlib
import io
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


class _Vertex:
    def __init__(self, data):
        self.data = data

    def __getitem__(self, k):
        return self.data[k]


class _PlyData:
    """The slice of plyfile.PlyData the reference's loader uses: read() of a
    binary little-endian file whose only element is `vertex`."""

    _TYPES = {"float": "<f4", "float32": "<f4", "double": "<f8", "uchar": "u1", "uint8": "u1"}

    def __init__(self, vertex):
        self._v = vertex

    def __getitem__(self, k):
        assert k == "vertex"
        return self._v

    @classmethod
    def read(cls, path):
        raw = Path(path).read_bytes()
        end = raw.index(b"end_header\n") + len(b"end_header\n")
        count, fields = 0, []
        for line in raw[:end].decode().splitlines():
            t = line.split()
            if t[:2] == ["element", "vertex"]:
                count = int(t[2])
            elif t and t[0] == "property":
                fields.append((t[2], cls._TYPES[t[1]]))
        return cls(_Vertex(np.frombuffer(raw[end:], np.dtype(fields), count)))


def _install_stand_ins() -> None:
    core = types.ModuleType("mlx.core")
    core.float32, core.int32 = np.float32, np.int32

    class array:  # a class: the script uses mx.array in annotations
        def __new__(cls, x, dtype=None):
            return np.array(x, dtype=dtype)

    core.array = array
    core.set_cache_limit = lambda *a, **k: None
    core.eval = lambda *a, **k: None
    nn = types.ModuleType("mlx.nn")

    class Module:
        def __init__(self):
            pass

    nn.Module = Module
    nn.value_and_grad = lambda *a, **k: None
    opt = types.ModuleType("mlx.optimizers")
    opt.Adam = object
    pkg = types.ModuleType("mlx")
    pkg.core, pkg.nn, pkg.optimizers = core, nn, opt
    ply = types.ModuleType("plyfile")
    ply.PlyData = _PlyData
    sys.modules.update({"mlx": pkg, "mlx.core": core, "mlx.nn": nn, "mlx.optimizers": opt,
                        "cv2": types.ModuleType("cv2"), "plyfile": ply})


def _ply_bytes(points, rgb) -> bytes:
    fields = [("x", "<f4"), ("y", "<f4"), ("z", "<f4")]
    props = "property float x\nproperty float y\nproperty float z\n"
    if rgb is not None:
        fields += [("red", "u1"), ("green", "u1"), ("blue", "u1")]
        props += "property uchar red\nproperty uchar green\nproperty uchar blue\n"
    arr = np.empty(len(points), np.dtype(fields))
    arr["x"], arr["y"], arr["z"] = points.T
    if rgb is not None:
        arr["red"], arr["green"], arr["blue"] = rgb.T
    head = (f"ply\nformat binary_little_endian 1.0\nelement vertex {len(points)}\n" + props
            + "end_header\n")
    return head.encode() + arr.tobytes()


def _rot(rng):
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


def make_capture(seed: int, frames: int, colours: bool) -> dict[str, bytes]:
    """File name -> bytes of a small seeded scanner capture."""
    from PIL import Image

    rng = np.random.default_rng(seed)
    files = {}
    pts = rng.normal(0, 1.5, (120, 3)).astype(np.float32)
    rgb = rng.integers(0, 256, (120, 3)).astype(np.uint8) if colours else None
    files["points.ply"] = _ply_bytes(pts, rgb)
    for i in range(frames):
        img = rng.integers(0, 256, (48, 64, 3)).astype(np.uint8)
        buf = io.BytesIO()
        Image.fromarray(img).save(buf, format="JPEG", quality=90)
        files[f"frame_{i:05d}.jpg"] = buf.getvalue()
        pose = np.eye(4)
        pose[:3, :3] = _rot(rng)
        pose[:3, 3] = rng.normal(0, 2.0, 3)
        k = [55.0 + i, 0.0, 31.0 + 0.5 * i, 0.0, 53.0 + i, 23.5, 0.0, 0.0, 1.0]
        files[f"frame_{i:05d}.json"] = json.dumps(
            {"intrinsics": k, "cameraPoseARFrame": pose.reshape(-1).tolist()}).encode()
    return files


# tag -> (seed, frames, colours, prepare_dataset keyword arguments)
CASES = {
    "plain": (1, 4, True, dict(width=32, height=24, max_frames=120, frame_step=1, start_index=0,
                                max_points=0, seed=42, extra_points_ratio=0.0,
                                extra_points_mode="surface-jitter", extra_points_jitter_scale=0.01)),
    "jitter": (2, 6, True, dict(width=40, height=30, max_frames=2, frame_step=2, start_index=1,
                                 max_points=90, seed=7, extra_points_ratio=0.5,
                                 extra_points_mode="surface-jitter", extra_points_jitter_scale=0.02)),
    "bbox": (3, 3, False, dict(width=64, height=48, max_frames=120, frame_step=1, start_index=0,
                                max_points=0, seed=3, extra_points_ratio=0.25,
                                extra_points_mode="bbox", extra_points_jitter_scale=0.01)),
}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=None)
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    from oracle.build import default_reference_dir

    ref_dir = a.reference_dir or default_reference_dir()
    _install_stand_ins()
    sys.path.insert(0, os.path.join(ref_dir, "scripts"))
    fixed = importlib.import_module("train_scanner_fixed")
    import tempfile

    out = {}
    for tag, (seed, frames, colours, kw) in CASES.items():
        files = make_capture(seed, frames, colours)
        for name, data in files.items():
            out[f"{tag}/file/{name}"] = np.frombuffer(data, np.uint8)
        with tempfile.TemporaryDirectory() as d:
            for name, data in files.items():
                (Path(d) / name).write_bytes(data)
            cams, targets, points, colors, base = fixed.prepare_dataset(dataset_dir=Path(d), **kw)
        out[f"{tag}/points"] = points
        out[f"{tag}/colors"] = np.asarray(colors, np.float32)
        out[f"{tag}/base"] = np.int64(base)
        for i, (c, t) in enumerate(zip(cams, targets)):
            out[f"{tag}/cam{i}/viewmatrix"] = np.asarray(c.viewmatrix, np.float32)
            out[f"{tag}/cam{i}/projmatrix"] = np.asarray(c.projmatrix, np.float32)
            out[f"{tag}/cam{i}/campos"] = np.asarray(c.campos, np.float32)
            out[f"{tag}/cam{i}/tan"] = np.array([c.tan_fovx, c.tan_fovy], np.float64)
            out[f"{tag}/cam{i}/size"] = np.array([c.image_width, c.image_height], np.int64)
            out[f"{tag}/cam{i}/target"] = np.asarray(t, np.float32)
        out[f"{tag}/ncams"] = np.int64(len(cams))
        model = fixed.init_model(points, np.asarray(colors, np.float32), 3)
        for k in ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales",
                  "rotations"):
            out[f"{tag}/init/{k}"] = np.asarray(getattr(model, k), np.float32)
    path = os.path.join(HERE, "dataset_ref.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, sum(v.nbytes for v in out.values()), "bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
