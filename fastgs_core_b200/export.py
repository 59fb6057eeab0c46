"""Export of a trained set of Gaussians:

* the arrays the reference hands to the spz library (save_as_spz,
  scripts/train_scanner_fixed.py:631-688): log-scales, opacity logits, dc
  and rest SH as stored, positions and rotations moved into the y-up frame
  of the Scaniverse preview ((x, y, z) -> (x, -z, y), rotations conjugated
  by the same axis change); save_as_spz writes them through the `spz`
  module when it is importable and otherwise returns False, as the
  reference does;
* the common 3DGS PLY layout (binary little endian; x y z, nx ny nz, f_dc_*,
  f_rest_* channel-major, opacity logit, scale_* (log), rot_* (w x y z)),
  written and read back.
"""
from __future__ import annotations

import numpy as np

from .synthetic import Scene

_AXIS = np.array([[1.0, 0.0, 0.0], [0.0, 0.0, 1.0], [0.0, -1.0, 0.0]], np.float32)


def quat_to_matrix(q: np.ndarray) -> np.ndarray:
    """Rotation matrices of w-first quaternions (normalised first)."""
    q = np.asarray(q, np.float32)
    q = q / np.clip(np.linalg.norm(q, axis=1, keepdims=True), 1.0e-8, None)
    w, x, y, z = q.T
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)], 1).astype(np.float32)


def matrix_to_quat(r: np.ndarray) -> np.ndarray:
    """w-first unit quaternions of rotation matrices: the branch on the
    largest of the trace and the diagonal entries keeps the square root's
    argument away from zero (Shepperd's method)."""
    r = np.asarray(r, np.float32)
    m = r.shape[0]
    q = np.empty((m, 4), np.float32)
    tr = r[:, 0, 0] + r[:, 1, 1] + r[:, 2, 2]
    c0 = tr > 0
    cx = ~c0 & (r[:, 0, 0] > r[:, 1, 1]) & (r[:, 0, 0] > r[:, 2, 2])
    cy = ~c0 & ~cx & (r[:, 1, 1] > r[:, 2, 2])
    cz = ~c0 & ~cx & ~cy
    s = np.sqrt(tr[c0] + 1.0) * 2.0
    q[c0] = np.stack([0.25 * s, (r[c0, 2, 1] - r[c0, 1, 2]) / s, (r[c0, 0, 2] - r[c0, 2, 0]) / s,
                      (r[c0, 1, 0] - r[c0, 0, 1]) / s], -1)
    s = np.sqrt(1.0 + r[cx, 0, 0] - r[cx, 1, 1] - r[cx, 2, 2]) * 2.0
    q[cx] = np.stack([(r[cx, 2, 1] - r[cx, 1, 2]) / s, 0.25 * s, (r[cx, 0, 1] + r[cx, 1, 0]) / s,
                      (r[cx, 0, 2] + r[cx, 2, 0]) / s], -1)
    s = np.sqrt(1.0 + r[cy, 1, 1] - r[cy, 0, 0] - r[cy, 2, 2]) * 2.0
    q[cy] = np.stack([(r[cy, 0, 2] - r[cy, 2, 0]) / s, (r[cy, 0, 1] + r[cy, 1, 0]) / s, 0.25 * s,
                      (r[cy, 1, 2] + r[cy, 2, 1]) / s], -1)
    s = np.sqrt(1.0 + r[cz, 2, 2] - r[cz, 0, 0] - r[cz, 1, 1]) * 2.0
    q[cz] = np.stack([(r[cz, 1, 0] - r[cz, 0, 1]) / s, (r[cz, 0, 2] + r[cz, 2, 0]) / s,
                      (r[cz, 1, 2] + r[cz, 2, 1]) / s, 0.25 * s], -1)
    return q / np.clip(np.linalg.norm(q, axis=1, keepdims=True), 1.0e-8, None)


def trainer_arrays(tr) -> dict:
    """The trainer's raw parameters as numpy arrays (scene layout)."""
    n = tr.n
    f = tr.params.detach().cpu().numpy()
    return {"means3d": f[:3 * n].reshape(n, 3), "features_dc": f[3 * n:6 * n].reshape(n, 3),
            "features_rest": f[6 * n:51 * n].reshape(n, 15, 3), "opacity_logits": f[51 * n:52 * n],
            "log_scales": f[52 * n:55 * n].reshape(n, 3), "rotations": f[55 * n:59 * n].reshape(n, 4)}


def spz_cloud_arrays(params: dict) -> dict:
    """What save_as_spz gives spz.GaussianCloud (flattened float32)."""
    m = params["means3d"]
    pos = np.stack([m[:, 0], -m[:, 2], m[:, 1]], -1)
    rot = matrix_to_quat(_AXIS @ quat_to_matrix(params["rotations"]) @ _AXIS.T)
    return {"positions": pos.reshape(-1).astype(np.float32),
            "scales": params["log_scales"].reshape(-1).astype(np.float32),
            "rotations": rot.reshape(-1).astype(np.float32),
            "alphas": params["opacity_logits"].reshape(-1).astype(np.float32),
            "colors": params["features_dc"].reshape(-1).astype(np.float32),
            "sh": params["features_rest"].reshape(-1).astype(np.float32)}


def save_as_spz(filename, tr, sh_degree: int) -> bool:
    """save_as_spz (scripts/train_scanner_fixed.py:631-688) for a Trainer."""
    try:
        import spz  # noqa: PLC0415
    except ImportError:
        print("[WARN] spz is not available; skip final.spz export")
        return False
    a = spz_cloud_arrays(trainer_arrays(tr))
    cloud = spz.GaussianCloud()
    cloud.antialiased = True
    for k, v in a.items():
        setattr(cloud, k, v)
    cloud.sh_degree = int(sh_degree)
    if not spz.save_spz(cloud, spz.PackOptions(), str(filename)):
        raise RuntimeError(f"failed to save spz to {filename}")
    return True


def _ply_fields(rest_count: int):
    names = ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"]
    names += [f"f_rest_{i}" for i in range(3 * rest_count)]
    names += ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    return names


def save_ply(filename, params: dict) -> None:
    """The common 3DGS PLY layout (binary little endian)."""
    n = params["means3d"].shape[0]
    rest = params["features_rest"]
    names = _ply_fields(rest.shape[1])
    cols = [params["means3d"], np.zeros((n, 3), np.float32), params["features_dc"],
            rest.transpose(0, 2, 1).reshape(n, -1),  # channel-major: all R, then G, then B
            params["opacity_logits"].reshape(n, 1), params["log_scales"], params["rotations"]]
    data = np.concatenate([np.asarray(c, np.float32).reshape(n, -1) for c in cols], 1)
    assert data.shape[1] == len(names)
    header = "ply\nformat binary_little_endian 1.0\nelement vertex %d\n" % n
    header += "".join(f"property float {nm}\n" for nm in names) + "end_header\n"
    with open(filename, "wb") as fh:
        fh.write(header.encode("ascii"))
        fh.write(data.astype("<f4").tobytes())


def load_ply(filename, sh_degree: int = 3) -> Scene:
    """Read save_ply's layout back into a Scene."""
    with open(filename, "rb") as fh:
        raw = fh.read()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    lines = raw[:end].decode("ascii").splitlines()
    n = int(next(ln.split()[2] for ln in lines if ln.startswith("element vertex")))
    names = [ln.split()[2] for ln in lines if ln.startswith("property")]
    data = np.frombuffer(raw[end:end + 4 * n * len(names)], "<f4").reshape(n, len(names))
    col = {nm: i for i, nm in enumerate(names)}

    def take(*ks):
        return np.ascontiguousarray(data[:, [col[k] for k in ks]], np.float32)

    rest_n = sum(1 for nm in names if nm.startswith("f_rest_")) // 3
    rest = take(*[f"f_rest_{i}" for i in range(3 * rest_n)]).reshape(n, 3, rest_n).transpose(0, 2, 1)
    return Scene(take("x", "y", "z"), take("f_dc_0", "f_dc_1", "f_dc_2"), np.ascontiguousarray(rest),
                 take("opacity")[:, 0].copy(), take("scale_0", "scale_1", "scale_2"),
                 take("rot_0", "rot_1", "rot_2", "rot_3"), sh_degree)
