"""Scanner dataset loader (no GPU): a two-frame dataset written here in the
reference's layout, loaded back."""
import json

import numpy as np
import pytest
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


def _golden_case(tag, tmp_path):
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "dataset_ref.npz"))
    pre = f"{tag}/file/"
    for k in z.files:
        if k.startswith(pre):
            (tmp_path / k[len(pre):]).write_bytes(z[k].tobytes())
    return z


# the keyword arguments tests/golden/make_dataset_golden.py gave the reference's prepare_dataset
_GOLDEN_KW = {
    "plain": dict(width=32, height=24, max_frames=120, frame_step=1, start_index=0, max_points=0,
                  seed=42, extra_points_ratio=0.0, extra_points_mode="surface-jitter",
                  extra_points_jitter_scale=0.01),
    "jitter": dict(width=40, height=30, max_frames=2, frame_step=2, start_index=1, max_points=90,
                   seed=7, extra_points_ratio=0.5, extra_points_mode="surface-jitter",
                   extra_points_jitter_scale=0.02),
    "bbox": dict(width=64, height=48, max_frames=120, frame_step=1, start_index=0, max_points=0,
                 seed=3, extra_points_ratio=0.25, extra_points_mode="bbox",
                 extra_points_jitter_scale=0.01),
}


@pytest.mark.parametrize("tag", sorted(_GOLDEN_KW))
def test_prepare_dataset_matches_reference_loader(tag, tmp_path):
    """The loader against the reference's own prepare_dataset / init_model run
    on the same capture (tests/golden/make_dataset_golden.py): frame selection,
    axis change and normalisation, subsampling and extra points from the same
    seeded draws, cameras, resized targets and the initial parameters."""
    z = _golden_case(tag, tmp_path)
    kw = dict(_GOLDEN_KW[tag])
    w, h = kw.pop("width"), kw.pop("height")
    cams, targets, points, colors, base = DS.prepare_dataset(tmp_path, w, h, **kw)
    assert base == int(z[f"{tag}/base"]) and len(cams) == int(z[f"{tag}/ncams"])
    np.testing.assert_array_equal(points, z[f"{tag}/points"])
    np.testing.assert_array_equal(colors, z[f"{tag}/colors"])
    for i, c in enumerate(cams):
        p = f"{tag}/cam{i}/"
        np.testing.assert_array_equal(np.asarray(c.viewmatrix, np.float32), z[p + "viewmatrix"])
        np.testing.assert_array_equal(np.asarray(c.projmatrix, np.float32), z[p + "projmatrix"])
        np.testing.assert_array_equal(np.asarray(c.campos, np.float32).reshape(-1),
                                      z[p + "campos"].reshape(-1))
        assert (c.tan_fovx, c.tan_fovy) == tuple(z[p + "tan"])
        assert (c.width, c.height) == tuple(z[p + "size"])
        np.testing.assert_allclose(targets[i], z[p + "target"], rtol=0, atol=1e-6)
    scene = DS.init_scene(points, colors, 3)
    for k in ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations"):
        np.testing.assert_array_equal(np.asarray(getattr(scene, k), np.float32), z[f"{tag}/init/{k}"])
