"""Export helpers (no GPU): PLY round trip and the spz frame change."""
import numpy as np

from fastgs_core_b200 import export as E
from fastgs_core_b200 import synthetic as S


def _params(scene):
    return {"means3d": scene.means3d, "features_dc": scene.features_dc,
            "features_rest": scene.features_rest, "opacity_logits": scene.opacity_logits,
            "log_scales": scene.log_scales, "rotations": scene.rotations}


def test_ply_round_trip(tmp_path):
    scene, _ = S.small_scene(2, 257, 3, 32, 32)
    p = tmp_path / "g.ply"
    E.save_ply(p, _params(scene))
    back = E.load_ply(p)
    for k, v in _params(scene).items():
        assert np.array_equal(getattr(back, k), v), k
    head = p.read_bytes()[:2000].decode("ascii", "ignore")
    assert "element vertex 257" in head and "property float f_rest_44" in head


def test_quaternion_matrix_round_trip():
    rng = np.random.default_rng(0)
    q = rng.normal(size=(1000, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    q[q[:, 0] < 0] *= -1
    back = E.matrix_to_quat(E.quat_to_matrix(q))
    back[back[:, 0] < 0] *= -1
    np.testing.assert_allclose(back, q, atol=2e-5)


def test_spz_frame_change():
    scene, _ = S.small_scene(3, 100, 3, 32, 32)
    a = E.spz_cloud_arrays(_params(scene))
    pos = a["positions"].reshape(-1, 3)
    assert np.array_equal(pos[:, 0], scene.means3d[:, 0])
    assert np.array_equal(pos[:, 1], -scene.means3d[:, 2])
    assert np.array_equal(pos[:, 2], scene.means3d[:, 1])
    # the rotation conjugated by the axis change: R' = A R A^T
    rm = E.quat_to_matrix(a["rotations"].reshape(-1, 4))
    want = E._AXIS @ E.quat_to_matrix(scene.rotations) @ E._AXIS.T
    np.testing.assert_allclose(rm, want, atol=3e-5)
    assert np.array_equal(a["scales"], scene.log_scales.reshape(-1))


def test_spz_known_bytes(tmp_path):
    """One hand-encoded point against the packed layout byte for byte."""
    import gzip
    import struct

    cloud = {"positions": np.array([1.0, -2.5, 0.000244140625], np.float32),
             "alphas": np.array([0.0], np.float32), "colors": np.array([0.0, 1.0, -1.0], np.float32),
             "scales": np.array([-4.0, -10.0, 6.0], np.float32),
             "rotations": np.array([0.0, 0.0, 0.0, -1.0], np.float32),  # x y z w; w < 0 flips
             "sh": np.array([0.5, -0.25, 0.0] * 3 + [1.0, -1.0, 0.1] * 5, np.float32)}
    p = tmp_path / "one.spz"
    E.write_spz(p, cloud, 2)
    raw = gzip.open(p, "rb").read()
    assert struct.unpack_from("<IIIBBBB", raw) == (0x5053474E, 2, 1, 2, 12, 1, 0)
    body = raw[16:]
    pos = body[:9]
    assert pos == bytes([0x00, 0x10, 0x00, 0x00, 0xD8, 0xFF, 0x01, 0x00, 0x00])  # 4096, -10240, 1
    assert body[9] == 128                                  # sigmoid(0) * 255 = 127.5 -> 128
    assert list(body[10:13]) == [128, 166, 89]             # 127.5 + c * 38.25, rounded
    assert list(body[13:16]) == [96, 0, 255]               # (s + 10) * 16, clamped
    assert list(body[16:19]) == [128, 128, 128]            # (0, 0, 0, 1) after the sign flip
    # degree 1 (9 values, buckets of 8), then 15 values in buckets of 16
    assert list(body[19:28]) == [192, 96, 128] * 3
    assert list(body[28:43]) == [255, 0, 144] * 5
    assert len(body) == 43


def test_spz_round_trip(tmp_path):
    scene, _ = S.small_scene(5, 500, 3, 32, 32)
    a = E.spz_cloud_arrays(_params(scene))
    p = tmp_path / "scene.spz"
    E.write_spz(p, a, 3)
    b = E.read_spz(p)
    assert b["sh_degree"] == 3 and b["antialiased"]
    np.testing.assert_allclose(b["positions"], a["positions"], atol=0.5 / 4096 + 1e-7)
    np.testing.assert_allclose(b["scales"], np.clip(a["scales"], -10, 255 / 16 - 10), atol=0.5 / 16 + 1e-6)
    np.testing.assert_allclose(b["colors"], np.clip(a["colors"], -127.5 / 38.25, 127.5 / 38.25),
                               atol=0.5 / 38.25 + 1e-6)
    op_a = 1 / (1 + np.exp(-a["alphas"]))
    op_b = 1 / (1 + np.exp(-b["alphas"].astype(np.float64)))
    np.testing.assert_allclose(op_b, op_a, atol=0.5 / 255 + 1e-6)
    qa = a["rotations"].reshape(-1, 4)
    qa = qa / np.linalg.norm(qa, axis=1, keepdims=True) * np.where(qa[:, 3:4] < 0, -1, 1)
    qb = b["rotations"].reshape(-1, 4)
    assert np.abs(qb[:, :3] - qa[:, :3]).max() <= 0.5 / 127.5 + 1e-6
    sh_a, sh_b = a["sh"].reshape(500, -1), b["sh"].reshape(500, -1)
    assert np.abs(sh_b[:, :9] - np.clip(sh_a[:, :9], -1, 127 / 128)).max() <= 4.5 / 128
    assert np.abs(sh_b[:, 9:] - np.clip(sh_a[:, 9:], -1, 127 / 128)).max() <= 8.5 / 128


def test_spz_cloud_matches_reference_exporter():
    """spz_cloud_arrays against what the reference's own save_as_spz hands to
    spz.GaussianCloud for the same model (tests/golden/make_export_golden.py):
    app-frame positions, raw log-scales, axis-conjugated rotations of the
    normalised quaternions, logits, dc and rest coefficients."""
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "export_ref.npz"))
    params = {k[3:]: z[k] for k in z.files if k.startswith("in/")}
    got = E.spz_cloud_arrays(params)
    for k in ("positions", "scales", "alphas", "colors", "sh"):
        np.testing.assert_array_equal(got[k], z["cloud/" + k].astype(np.float32), err_msg=k)
    # a quaternion and its negation are the same rotation
    q, w = got["rotations"].reshape(-1, 4), z["cloud/rotations"].reshape(-1, 4)
    sgn = np.where((q * w).sum(1, keepdims=True) < 0, -1.0, 1.0)
    np.testing.assert_allclose(q * sgn, w, rtol=0, atol=2e-6)
    assert int(z["cloud/sh_degree"]) == 3
