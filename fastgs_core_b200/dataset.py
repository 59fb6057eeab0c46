"""The scanner dataset loader of the reference's training scripts
(prepare_dataset, scripts/train_scanner_fixed.py:237-598): frame_<i>.jpg /
frame_<i>.json pairs (intrinsics [9], cameraPoseARFrame [16]) and points.ply,
moved into the training frame ((x, y, z) -> (x, z, -y)), normalised by the
camera centres, and the cameras built as the rasterizer expects them
(view = W2C^T, full projection = (P W2C)^T). init_scene is init_model
(:601-628). Returns fastgs_core_b200.synthetic Camera / Scene objects and CHW
float32 targets.
"""
from __future__ import annotations

import json
import math
import re
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .synthetic import Camera, Scene


@dataclass
class ScannerFrame:
    index: int
    image_path: Path
    json_path: Path
    frame: dict | None = None


def make_axis_transform():
    """:301-312."""
    a = np.array([[1.0, 0.0, 0.0], [0.0, 0.0, 1.0], [0.0, -1.0, 0.0]], np.float32)
    a4 = np.eye(4, dtype=np.float32)
    a4[:3, :3] = a
    return a, a4


def read_ply_vertices(path) -> tuple[np.ndarray, np.ndarray | None]:
    """x, y, z (and red, green, blue if present, scaled to [0, 1]) of the
    vertex element of an ascii or binary little-endian PLY file
    (load_ply_positions_colors, :237-256)."""
    raw = Path(path).read_bytes()
    end = raw.index(b"end_header") + len(b"end_header")
    end = raw.index(b"\n", end) + 1
    header = raw[:end].decode("ascii").splitlines()
    fmt = next(ln.split()[1] for ln in header if ln.startswith("format"))
    types = {"char": "i1", "uchar": "u1", "int8": "i1", "uint8": "u1", "short": "i2", "ushort": "u2",
             "int16": "i2", "uint16": "u2", "int": "i4", "uint": "u4", "int32": "i4", "uint32": "u4",
             "float": "f4", "float32": "f4", "double": "f8", "float64": "f8"}
    n, props, in_vertex = 0, [], False
    for ln in header:
        p = ln.split()
        if p[:1] == ["element"]:
            in_vertex = p[1] == "vertex"
            if in_vertex:
                n = int(p[2])
        elif p[:1] == ["property"] and in_vertex:
            if p[1] == "list":
                raise ValueError("list properties in the vertex element are not supported")
            props.append((p[2], types[p[1]]))
    if fmt == "ascii":
        rows = raw[end:].decode("ascii").split("\n")[:n]
        data = np.array([[float(x) for x in r.split()[:len(props)]] for r in rows], np.float64)
        col = {nm: data[:, i] for i, (nm, _) in enumerate(props)}
    elif fmt == "binary_little_endian":
        dt = np.dtype([(nm, "<" + t) for nm, t in props])
        arr = np.frombuffer(raw[end:end + n * dt.itemsize], dt)
        col = {nm: arr[nm] for nm, _ in props}
    else:
        raise ValueError(f"unsupported PLY format {fmt}")
    points = np.stack([col["x"], col["y"], col["z"]], 1).astype(np.float32)
    colors = None
    if all(k in col for k in ("red", "green", "blue")):
        colors = np.stack([col["red"], col["green"], col["blue"]], 1).astype(np.float32)
        if colors.max() > 1.0:
            colors = colors / 255.0
        colors = np.clip(colors, 0.0, 1.0)
    return points, colors


def collect_scanner_frames(dataset_dir, max_frames: int, frame_step: int, start_index: int):
    """:264-298."""
    d = Path(dataset_dir)

    def index(p):
        m = re.search(r"frame_(\d+)", p.stem)
        return None if m is None else int(m.group(1))

    images = {index(p): p for p in sorted(d.glob("frame_*.jpg")) if index(p) is not None}
    jsons = {index(p): p for p in sorted(d.glob("frame_*.json")) if index(p) is not None}
    common = [i for i in sorted(set(images) & set(jsons)) if i >= start_index]
    if frame_step > 1:
        common = common[::frame_step]
    if max_frames > 0:
        common = common[:max_frames]
    if not common:
        raise RuntimeError(f"No scanner frame pairs found in {dataset_dir}")
    return [ScannerFrame(i, images[i], jsons[i]) for i in common]


def compute_normalization(camera_positions):
    """:315-320."""
    c = np.stack(camera_positions, 0).astype(np.float32)
    t = c.mean(axis=0)
    denom = np.max(np.abs(c - t[None, :]))
    return t, (1.0 / float(denom) if denom > 0.0 else 1.0)


def build_camera_from_scanner_json(frame: dict, width: int, height: int, znear: float = 0.001,
                                   zfar: float = 1000.0) -> Camera:
    """:323-385: pinhole intrinsics scaled to the render size, camera-to-world
    with the y and z axes flipped, OpenGL-style frustum projection."""
    w, h = float(width), float(height)
    sx, sy = w / float(frame.get("w", width)), h / float(frame.get("h", height))
    fx, fy = float(frame["fl_x"]) * sx, float(frame["fl_y"]) * sy
    c2w = np.array(frame["transform_matrix"], np.float32)
    r = c2w[:3, :3] @ np.diag([1.0, -1.0, -1.0]).astype(np.float32)
    t = c2w[:3, 3:4]
    rinv = r.T
    view = np.eye(4, dtype=np.float32)
    view[:3, :3] = rinv
    view[:3, 3:4] = -rinv @ t
    fovx, fovy = 2.0 * math.atan(w / (2.0 * fx)), 2.0 * math.atan(h / (2.0 * fy))
    top = znear * math.tan(0.5 * fovy)
    right = znear * math.tan(0.5 * fovx)
    proj = np.array([[2.0 * znear / (2 * right), 0.0, 0.0, 0.0],
                     [0.0, 2.0 * znear / (2 * top), 0.0, 0.0],
                     [0.0, 0.0, (zfar + znear) / (zfar - znear), -(zfar * znear) / (zfar - znear)],
                     [0.0, 0.0, 1.0, 0.0]], np.float32)
    full = proj @ view
    return Camera(int(width), int(height), math.tan(0.5 * fovx), math.tan(0.5 * fovy),
                  np.ascontiguousarray(view.T), np.ascontiguousarray(full.T),
                  t[:, 0].astype(np.float32).copy())


def load_target_image(path, width: int, height: int) -> np.ndarray:
    """:388-400: RGBA composited on white, bilinear resize; returns CHW."""
    from PIL import Image  # noqa: PLC0415

    with Image.open(path) as im:
        rgba = im.convert("RGBA")
        if rgba.size != (width, height):
            rgba = rgba.resize((width, height), Image.Resampling.BILINEAR)
        a = np.asarray(rgba, np.float32) / 255.0
    rgb = a[:, :, :3] * a[:, :, 3:4] + (1.0 - a[:, :, 3:4])
    return np.ascontiguousarray(rgb.transpose(2, 0, 1))


def prepare_dataset(dataset_dir, width: int, height: int, max_frames: int = 120, frame_step: int = 1,
                    start_index: int = 0, max_points: int = 30000000, seed: int = 42,
                    extra_points_ratio: float = 0.0, extra_points_mode: str = "surface-jitter",
                    extra_points_jitter_scale: float = 0.01):
    """:403-598. Returns cameras, CHW targets, points, colours, base point count."""
    from PIL import Image  # noqa: PLC0415

    a, a4 = make_axis_transform()
    frames = collect_scanner_frames(dataset_dir, max_frames, frame_step, start_index)
    points, colors = read_ply_vertices(Path(dataset_dir) / "points.ply")
    points = (a @ points.T).T
    positions = []
    for f in frames:
        raw = json.loads(Path(f.json_path).read_text(encoding="utf-8"))
        with Image.open(f.image_path) as im:
            rw, rh = im.size
        k = raw.get("intrinsics")
        if k is None or len(k) != 9:
            raise RuntimeError(f"Invalid intrinsics in {f.json_path}")
        pose = raw.get("cameraPoseARFrame")
        if pose is None or len(pose) != 16:
            raise RuntimeError(f"Invalid cameraPoseARFrame in {f.json_path}")
        c2w = (a4 @ np.array(pose, np.float32).reshape(4, 4)).astype(np.float32)
        f.frame = {"w": int(rw), "h": int(rh), "file_path": f.image_path.name, "fl_x": float(k[0]),
                   "fl_y": float(k[4]), "cx": float(k[2]), "cy": float(k[5]),
                   "transform_matrix": c2w.tolist()}
        positions.append(c2w[:3, 3])
    translation, scale = compute_normalization(positions)
    points = (points - translation[None, :]) * scale
    rng = np.random.default_rng(seed)
    if max_points > 0 and points.shape[0] > max_points:
        keep = rng.choice(points.shape[0], size=max_points, replace=False)
        points = points[keep]
        if colors is not None:
            colors = colors[keep]
    colors = colors.astype(np.float32) if colors is not None else np.full_like(points, 0.5, np.float32)
    base = int(points.shape[0])
    extra = int(round(points.shape[0] * extra_points_ratio))
    if extra > 0:
        lo, hi = points.min(axis=0), points.max(axis=0)
        if extra_points_mode == "surface-jitter":
            src = rng.integers(0, points.shape[0], size=extra)
            std = extra_points_jitter_scale * float(np.linalg.norm(hi - lo))
            xyz = points[src] + rng.normal(0.0, std, (extra, 3)).astype(np.float32)
            rgb = colors[src]
        elif extra_points_mode == "bbox":
            xyz = rng.uniform(low=lo, high=hi, size=(extra, 3)).astype(np.float32)
            rgb = colors[rng.integers(0, colors.shape[0], size=extra)]
        else:
            raise ValueError(f"Unsupported --extra-points-mode: {extra_points_mode}")
        points = np.concatenate([points, xyz], 0).astype(np.float32)
        colors = np.concatenate([colors, rgb.astype(np.float32)], 0)
    cameras, targets = [], []
    for f in frames:
        c2w = np.array(f.frame["transform_matrix"], np.float32)
        c2w[:3, 3] = (c2w[:3, 3] - translation) * scale
        fr = dict(f.frame)
        fr["transform_matrix"] = c2w.tolist()
        cameras.append(build_camera_from_scanner_json(fr, width, height))
        targets.append(load_target_image(f.image_path, width, height))
    return cameras, targets, points.astype(np.float32), colors, base


def init_scene(points: np.ndarray, colors: np.ndarray, sh_degree: int = 3) -> Scene:
    """init_model (:601-628): scale 0.02, identity rotation, opacity 0.82, dc
    from the point colours, zero higher SH bands."""
    n = points.shape[0]
    log_scales = np.full((n, 3), math.log(0.02), np.float32)
    rotations = np.zeros((n, 4), np.float32)
    rotations[:, 0] = 1.0
    p = np.clip(np.full(n, 0.82, np.float32), 1.0e-6, 1.0 - 1.0e-6)
    opacity_logits = np.log(p / (1.0 - p)).astype(np.float32)
    dc = ((colors - 0.5) / 0.28209479177387814).astype(np.float32)
    rest = np.zeros((n, max(0, (sh_degree + 1) ** 2 - 1), 3), np.float32)
    return Scene(np.ascontiguousarray(points, np.float32), dc, rest, opacity_logits, log_scales,
                 rotations, sh_degree)
