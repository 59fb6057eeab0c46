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
