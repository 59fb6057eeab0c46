"""Export of a trained set of Gaussians:

* the arrays the reference hands to the spz library (save_as_spz,
  scripts/train_scanner_fixed.py:631-688): log-scales, opacity logits, dc
  and rest SH as stored, positions and rotations moved into the y-up frame
  of the Scaniverse preview ((x, y, z) -> (x, -z, y), rotations conjugated
  by the same axis change), written by this module's own .spz encoder
  (write_spz), since the reference's `spz` submodule (nianticlabs/spz,
  .gitmodules:1-3) is not part of its tree; read_spz decodes the files;
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


# ------------------------------------------------------------------ .spz
# The packed Gaussian format of nianticlabs/spz (version 2 of its published
# layout): a gzip stream holding a 16-byte little-endian header
#   uint32 magic 0x5053474e ("NGSP"), uint32 version, uint32 point count,
#   uint8 SH degree, uint8 fractional bits, uint8 flags (1 = antialiased),
#   uint8 reserved
# followed by one block per attribute, points in order:
#   positions  3 x 24-bit two's complement fixed point (round(x * 2^bits))
#   alphas     uint8 round(sigmoid(logit) * 255)
#   colors     3 x uint8 round(dc * 0.15 * 255 + 127.5)
#   scales     3 x uint8 round((log_scale + 10) * 16)
#   rotations  3 x uint8 of the unit quaternion (x, y, z, w) with w >= 0:
#              round(v * 127.5 + 127.5) for x, y, z (w is recovered)
#   sh         (coefficient, channel) x uint8 q = round(v * 128) + 128,
#              rounded to buckets of 8 (the 9 values of degree 1) or 16
#              (higher degrees)
# uint8 quantities are clamped to [0, 255].
SPZ_MAGIC = 0x5053474E
SPZ_VERSION = 2
SPZ_FRACTIONAL_BITS = 12
_SPZ_COLOR_SCALE = 0.15


def _round(x) -> np.ndarray:
    """Round half away from zero (C's round / lround, which the format's
    encoder uses), in float32 arithmetic like the encoder."""
    x = np.asarray(x, np.float32)
    return np.sign(x) * np.floor(np.abs(x) + np.float32(0.5))


def _u8(x) -> np.ndarray:
    return np.clip(_round(x), 0, 255).astype(np.uint8)


def _sh_quantize(x, bucket: int) -> np.ndarray:
    q = (_round(np.asarray(x, np.float32) * np.float32(128.0)) + 128.0).astype(np.int64)
    q = (q + bucket // 2) // bucket * bucket
    return np.clip(q, 0, 255).astype(np.uint8)


def _sh_dim(degree: int) -> int:
    return (degree + 1) ** 2 - 1


def write_spz(filename, cloud: dict, sh_degree: int, antialiased: bool = True) -> None:
    """Write the spz_cloud_arrays dictionary (flat float32 arrays of the
    spz.GaussianCloud fields; rotations as given, read as x, y, z, w) to a
    .spz file."""
    import gzip
    import struct

    pos = np.asarray(cloud["positions"], np.float32).reshape(-1, 3)
    n = pos.shape[0]
    dim = _sh_dim(int(sh_degree))
    sh = np.asarray(cloud.get("sh", np.zeros(0, np.float32)), np.float32).reshape(n, -1)
    if sh.shape[1] < 3 * dim:
        raise ValueError(f"sh holds {sh.shape[1] // 3} coefficients per point, degree {sh_degree} "
                         f"needs {dim}")
    sh = sh[:, :3 * dim]
    f32 = np.float32
    fixed = _round(pos * f32(1 << SPZ_FRACTIONAL_BITS)).astype(np.int64)
    fixed = np.clip(fixed, -(1 << 23), (1 << 23) - 1) & 0xFFFFFF
    pos_b = np.stack([(fixed >> (8 * k)) & 0xFF for k in range(3)], -1).astype(np.uint8)
    logits = np.asarray(cloud["alphas"], f32).reshape(n)
    alpha_b = _u8((f32(1.0) / (f32(1.0) + np.exp(-logits))) * f32(255.0))
    color_b = _u8(np.asarray(cloud["colors"], f32).reshape(n, 3) * f32(_SPZ_COLOR_SCALE * 255.0)
                  + f32(0.5 * 255.0))
    scale_b = _u8((np.asarray(cloud["scales"], f32).reshape(n, 3) + f32(10.0)) * f32(16.0))
    q = np.asarray(cloud["rotations"], f32).reshape(n, 4)
    q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), f32(1e-30))
    q = q * np.where(q[:, 3:4] < 0, f32(-127.5), f32(127.5)) + f32(127.5)
    rot_b = _u8(q[:, :3])
    sh_b = np.empty((n, 3 * dim), np.uint8)
    k1 = min(9, 3 * dim)
    sh_b[:, :k1] = _sh_quantize(sh[:, :k1], 8)
    sh_b[:, k1:] = _sh_quantize(sh[:, k1:], 16)
    header = struct.pack("<IIIBBBB", SPZ_MAGIC, SPZ_VERSION, n, int(sh_degree), SPZ_FRACTIONAL_BITS,
                         1 if antialiased else 0, 0)
    body = b"".join(a.tobytes() for a in (pos_b, alpha_b, color_b, scale_b, rot_b, sh_b))
    with gzip.open(filename, "wb") as fh:
        fh.write(header + body)


def read_spz(filename) -> dict:
    """Decode a .spz file (versions 2 and 3 of the packed layout) into the
    spz_cloud_arrays fields plus sh_degree and antialiased."""
    import gzip
    import struct

    with gzip.open(filename, "rb") as fh:
        raw = fh.read()
    magic, version, n, deg, bits, flags, _ = struct.unpack_from("<IIIBBBB", raw, 0)
    if magic != SPZ_MAGIC:
        raise ValueError(f"{filename}: not an spz file (magic {magic:#x})")
    if version not in (2, 3):
        raise ValueError(f"{filename}: unsupported spz version {version}")
    dim = _sh_dim(deg)
    off = 16

    def take(count):
        nonlocal off
        a = np.frombuffer(raw, np.uint8, count, off)
        off += count
        return a

    pb = take(9 * n).reshape(n, 3, 3).astype(np.int64)
    fixed = pb[..., 0] | (pb[..., 1] << 8) | (pb[..., 2] << 16)
    fixed = np.where(fixed & 0x800000, fixed - (1 << 24), fixed)
    positions = (fixed / float(1 << bits)).astype(np.float32)
    alphas_u = take(n).astype(np.float64) / 255.0
    alphas = np.log(np.clip(alphas_u, 1e-6, 1 - 1e-6) / np.clip(1 - alphas_u, 1e-6, None))
    colors = (take(3 * n).astype(np.float64) - 127.5) / (_SPZ_COLOR_SCALE * 255.0)
    scales = take(3 * n).astype(np.float64) / 16.0 - 10.0
    if version == 2:
        xyz = take(3 * n).reshape(n, 3).astype(np.float64) / 127.5 - 1.0
        w = np.sqrt(np.maximum(0.0, 1.0 - (xyz * xyz).sum(1, keepdims=True)))
        rotations = np.concatenate([xyz, w], 1)
    else:
        # smallest three: 2 bits of the largest component, 3 x 10 bits (sign + 9)
        packed = take(4 * n).reshape(n, 4).astype(np.uint32)
        v = packed[:, 0] | (packed[:, 1] << 8) | (packed[:, 2] << 16) | (packed[:, 3] << 24)
        largest = (v >> 30) & 3
        rotations = np.zeros((n, 4))
        mag_mask = (1 << 9) - 1
        rest = v.copy()
        sumsq = np.zeros(n)
        for i in range(3, -1, -1):
            sel = largest != i
            mag = (rest & mag_mask).astype(np.float64)
            neg = (rest >> 9) & 1
            comp = np.sqrt(0.5) * mag / mag_mask * np.where(neg == 1, -1.0, 1.0)
            rotations[sel, i] = comp[sel]
            sumsq += np.where(sel, comp * comp, 0.0)
            rest = np.where(sel, rest >> 10, rest)
        rotations[np.arange(n), largest] = np.sqrt(np.maximum(0.0, 1.0 - sumsq))
    sh = (take(3 * dim * n).astype(np.float64) - 128.0) / 128.0
    return {"positions": positions.reshape(-1), "alphas": alphas.astype(np.float32),
            "colors": colors.astype(np.float32).reshape(-1), "scales": scales.astype(np.float32).reshape(-1),
            "rotations": rotations.astype(np.float32).reshape(-1), "sh": sh.astype(np.float32),
            "sh_degree": int(deg), "antialiased": bool(flags & 1)}


def save_as_spz(filename, tr, sh_degree: int) -> bool:
    """save_as_spz (scripts/train_scanner_fixed.py:631-688) for a Trainer:
    the same arrays, antialiased, through write_spz."""
    write_spz(filename, spz_cloud_arrays(trainer_arrays(tr)), sh_degree, antialiased=True)
    print(f"saved spz: {filename}")
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
