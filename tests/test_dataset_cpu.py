"""Scanner dataset loader (no GPU): a two-frame dataset written here in the
reference's layout, loaded back."""
import json

import numpy as np
from PIL import Image

from fastgs_core_b200 import dataset as DS


def _write_dataset(d):
    rng = np.random.default_rng(0)
    pts = rng.normal(size=(50, 3)).astype(np.float32)
    rgb = rng.integers(0, 256, (50, 3)).astype(np.uint8)
    dt = np.dtype([("x", "<f4"), ("y", "<f4"), ("z", "<f4"), ("red", "u1"), ("green", "u1"), ("blue", "u1")])
    arr = np.empty(50, dt)
    arr["x"], arr["y"], arr["z"] = pts.T
    arr["red"], arr["green"], arr["blue"] = rgb.T
    head = ("ply\nformat binary_little_endian 1.0\nelement vertex 50\nproperty float x\n"
            "property float y\nproperty float z\nproperty uchar red\nproperty uchar green\n"
            "property uchar blue\nend_header\n")
    (d / "points.ply").write_bytes(head.encode() + arr.tobytes())
    for i, tx in enumerate((0.0, 2.0)):
        Image.fromarray(rng.integers(0, 256, (40, 60, 3)).astype(np.uint8)).save(d / f"frame_{i:05d}.jpg")
        pose = np.eye(4, dtype=np.float32)
        pose[0, 3] = tx
        (d / f"frame_{i:05d}.json").write_text(json.dumps(
            {"intrinsics": [50.0, 0, 30.0, 0, 50.0, 20.0, 0, 0, 1], "cameraPoseARFrame": pose.reshape(-1).tolist()}))
    return pts, rgb


def test_prepare_dataset(tmp_path):
    pts, rgb = _write_dataset(tmp_path)
    cams, targets, points, colors, base = DS.prepare_dataset(tmp_path, 30, 20)
    assert len(cams) == 2 and base == 50
    assert targets[0].shape == (3, 20, 30) and targets[0].dtype == np.float32
    # axis change and normalisation by the camera centres (x at 0 and 2: mean 1, half-range 1)
    a, _ = DS.make_axis_transform()
    want = ((a @ pts.T).T - np.array([1.0, 0.0, 0.0], np.float32)) * 1.0
    np.testing.assert_allclose(points, want, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(colors, rgb / 255.0, rtol=1e-6)
    c = cams[1]
    assert c.width == 30 and c.height == 20
    np.testing.assert_allclose(c.campos, [1.0, 0.0, 0.0], atol=1e-6)
    # fov from the intrinsics scaled to the render size (fx = 50 * 30 / 60)
    np.testing.assert_allclose(c.tan_fovx, 30 / (2 * 25.0), rtol=1e-6)
    # the view matrix (stored transposed) maps the camera centre to the origin
    v = c.viewmatrix.T
    np.testing.assert_allclose(v @ np.array([1.0, 0.0, 0.0, 1.0]), [0, 0, 0, 1], atol=1e-6)
    scene = DS.init_scene(points, colors, 3)
    assert scene.features_rest.shape == (50, 15, 3)
    np.testing.assert_allclose(scene.features_dc * 0.28209479177387814 + 0.5, colors, atol=1e-6)
