"""Seeded synthetic scenes and cameras for the benchmark configurations.

No public dataset is involved: every configuration is a seeded draw with the
shapes, sizes and value distributions of the five workloads the benchmark is
quoted on (means, log-scales, quaternions, opacity logits, SH coefficients,
camera placement, image size, field of view).

Camera matrices follow the reference's look-at construction
(scripts/render_2048_cube_smoke.py:56-104): ``viewmatrix`` is the world-to-view
matrix transposed and ``projmatrix`` is ``viewmatrix @ projection.T``, both
stored row-major and read column-major by the kernels; ``tan_fov`` is the
tangent of half the field of view; near 0.01, far 100.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

SH_C0 = 0.28209479177387814


@dataclass
class Camera:
    width: int
    height: int
    tan_fovx: float
    tan_fovy: float
    viewmatrix: np.ndarray  # [4,4] float32
    projmatrix: np.ndarray  # [4,4] float32
    campos: np.ndarray  # [3] float32


def _normalize(v: np.ndarray) -> np.ndarray:
    return v / np.linalg.norm(v)


def projection_matrix(znear: float, zfar: float, fovx: float, fovy: float) -> np.ndarray:
    """Perspective matrix of scripts/render_2048_cube_smoke.py:56-74."""
    tan_y = math.tan(fovy / 2.0)
    tan_x = math.tan(fovx / 2.0)
    top, right = tan_y * znear, tan_x * znear
    bottom, left = -top, -right
    p = np.zeros((4, 4), dtype=np.float32)
    p[0, 0] = 2.0 * znear / (right - left)
    p[1, 1] = 2.0 * znear / (top - bottom)
    p[0, 2] = (right + left) / (right - left)
    p[1, 2] = (top + bottom) / (top - bottom)
    p[3, 2] = 1.0
    p[2, 2] = zfar / (zfar - znear)
    p[2, 3] = -(zfar * znear) / (zfar - znear)
    return p


def look_at_camera(eye, target, width: int, height: int, fovy_deg: float,
                   up=(0.0, 1.0, 0.0), znear: float = 0.01, zfar: float = 100.0) -> Camera:
    """Camera at ``eye`` looking at ``target`` with vertical FOV ``fovy_deg``;
    the horizontal FOV follows from the aspect ratio."""
    fovy = math.radians(fovy_deg)
    fovx = 2.0 * math.atan(math.tan(fovy / 2.0) * width / height)
    eye = np.asarray(eye, dtype=np.float32)
    target = np.asarray(target, dtype=np.float32)
    up = np.asarray(up, dtype=np.float32)
    forward = _normalize(target - eye)
    right = _normalize(np.cross(forward, up))
    true_up = _normalize(np.cross(right, forward))
    w2v = np.eye(4, dtype=np.float32)
    w2v[0, :3] = right
    w2v[1, :3] = true_up
    w2v[2, :3] = forward
    w2v[:3, 3] = -w2v[:3, :3] @ eye
    world_view = w2v.T
    full_proj = world_view @ projection_matrix(znear, zfar, fovx, fovy).T
    return Camera(width, height, math.tan(fovx / 2.0), math.tan(fovy / 2.0),
                  np.ascontiguousarray(world_view, dtype=np.float32),
                  np.ascontiguousarray(full_proj, dtype=np.float32), eye.astype(np.float32))


def _random_quats(rng: np.random.Generator, n: int) -> np.ndarray:
    q = rng.standard_normal((n, 4)).astype(np.float32)
    return q / np.linalg.norm(q, axis=1, keepdims=True)


@dataclass
class Scene:
    """Raw (trainable) parameters, as the training scripts store them."""

    means3d: np.ndarray  # [N,3]
    features_dc: np.ndarray  # [N,3]
    features_rest: np.ndarray  # [N,S,3]
    opacity_logits: np.ndarray  # [N]
    log_scales: np.ndarray  # [N,3]
    rotations: np.ndarray  # [N,4] unit quaternions, w first
    sh_degree: int

    @property
    def n(self) -> int:
        return self.means3d.shape[0]

    def activated(self) -> dict:
        """Activated inputs (sigmoid / exp / normalise, as the reference
        trainers' getters do in scripts/train_scanner_fixed.py:523-535)."""
        q = self.rotations / (np.linalg.norm(self.rotations, axis=1, keepdims=True) + 1e-8)
        return dict(means3d=self.means3d, dc=self.features_dc, sh=self.features_rest,
                    opacities=(1.0 / (1.0 + np.exp(-self.opacity_logits))).astype(np.float32),
                    scales=np.exp(self.log_scales).astype(np.float32),
                    rotations=q.astype(np.float32))


def _sh(rng, n, degree, dc_raw_uniform: bool):
    s = (degree + 1) ** 2 - 1
    dc = rng.uniform(0.0, 1.0, (n, 3)).astype(np.float32)
    rest = (rng.normal(0.0, 0.05, (n, s, 3)) if s else np.zeros((n, 0, 3))).astype(np.float32)
    return dc, rest


def config1(seed: int = 0):
    """2048 Gaussians, 256x256, SH 0 (the reference's 2048-Gaussian cube smoke scale)."""
    rng = np.random.default_rng(seed)
    n = 2048
    means = rng.uniform(-1, 1, (n, 3)).astype(np.float32)
    log_scales = rng.normal(-3.5, 0.3, (n, 3)).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(0.0, 1.0, n).astype(np.float32)
    dc, rest = _sh(rng, n, 0, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, 0)
    cam = look_at_camera((0.0, 0.0, 4.0), (0.0, 0.0, 0.0), 256, 256, 60.0)
    return scene, [cam]


def _sphere_dir(rng):
    v = rng.standard_normal(3)
    return v / np.linalg.norm(v)


def config2(seed: int = 0, n: int = 100_000):
    """100k Gaussians, 800x800, SH 3, camera on a radius-5 sphere."""
    rng = np.random.default_rng(seed)
    means = rng.normal(0.0, 1.0, (n, 3)).astype(np.float32)
    log_scales = rng.normal(-4.5, 0.5, (n, 3)).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(-1.0, 1.5, n).astype(np.float32)
    dc, rest = _sh(rng, n, 3, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, 3)
    cam = look_at_camera(5.0 * _sphere_dir(rng), (0, 0, 0), 800, 800, 50.0)
    return scene, [cam]


def config3(seed: int = 0, n: int = 1_000_000, width: int = 1920, height: int = 1080):
    """1M Gaussians from a 64-component mixture, 1920x1080, SH 3, orbit radius 6."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-4, 4, (64, 3))
    comp = rng.integers(0, 64, n)
    means = (centres[comp] + rng.normal(0.0, 0.3, (n, 3))).astype(np.float32)
    log_scales = rng.normal(-4.5, 0.5, (n, 3)).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(-1.0, 1.5, n).astype(np.float32)
    dc, rest = _sh(rng, n, 3, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, 3)
    return scene, orbit_cameras(rng, 8, 6.0, 0.0, width, height, 65.0)


def orbit_cameras(rng, count, radius, height_jitter, width, height, fovy_deg, jitter=True):
    cams = []
    for k in range(count):
        a = 2.0 * math.pi * k / count + (rng.uniform(-0.2, 0.2) if jitter else 0.0)
        h = rng.uniform(-height_jitter, height_jitter) if height_jitter else 0.0
        eye = (radius * math.cos(a), h + 0.5, radius * math.sin(a))
        cams.append(look_at_camera(eye, (0, 0, 0), width, height, fovy_deg))
    return cams


def config4(seed: int = 0, n: int = 3_000_000):
    """3M Gaussians from a 256-component anisotropic mixture, 1600x1064, 8 views per step."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-8, 8, (256, 3))
    sig = rng.uniform(0.1, 0.6, (256, 3))
    comp = rng.integers(0, 256, n)
    means = (centres[comp] + rng.standard_normal((n, 3)) * sig[comp]).astype(np.float32)
    log_scales = rng.normal(-4.0, 0.6, (n, 3)).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(0.0, 1.5, n).astype(np.float32)
    dc, rest = _sh(rng, n, 3, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, 3)
    return scene, orbit_cameras(rng, 8, 10.0, 2.0, 1600, 1064, 60.0)


def config5(seed: int = 0, n: int = 6_000_000):
    """6M Gaussians, 10% large splats, 3840x2160 at distance 5, 70 degree FOV."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-3, 3, (n, 3)).astype(np.float32)
    big = rng.uniform(0, 1, n) < 0.1
    log_scales = np.where(big[:, None], rng.normal(-1.5, 0.3, (n, 3)),
                          rng.normal(-5.0, 0.3, (n, 3))).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(1.0, 1.0, n).astype(np.float32)
    dc, rest = _sh(rng, n, 3, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, 3)
    cam = look_at_camera((0.0, 0.0, 5.0), (0, 0, 0), 3840, 2160, 70.0)
    return scene, [cam]


def small_scene(seed: int, n: int, degree: int, width: int, height: int, spread: float = 1.0,
                log_scale_mu: float = -3.0, op_mu: float = 0.0):
    """Small randomized scene for parity tests (sizes the CPU checkers finish in seconds)."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-spread, spread, (n, 3)).astype(np.float32)
    log_scales = rng.normal(log_scale_mu, 0.4, (n, 3)).astype(np.float32)
    quats = _random_quats(rng, n)
    op_logits = rng.normal(op_mu, 1.5, n).astype(np.float32)
    dc, rest = _sh(rng, n, degree, True)
    scene = Scene(means, dc, rest, op_logits, log_scales, quats, degree)
    eye = 4.0 * _sphere_dir(rng)
    cam = look_at_camera(eye, (0, 0, 0), width, height, 55.0)
    return scene, cam


def render_inputs(scene: Scene, cam: Camera, background=(0.0, 0.0, 0.0)) -> dict:
    """Input dict in the rasterize_gaussians schema (numpy)."""
    a = scene.activated()
    n = scene.n
    return dict(means3d=a["means3d"], dc=a["dc"], sh=a["sh"], opacities=a["opacities"],
                scales=a["scales"], rotations=a["rotations"], viewmatrix=cam.viewmatrix,
                projmatrix=cam.projmatrix, campos=cam.campos.reshape(1, 3),
                background=np.asarray(background, np.float32),
                metric_map=np.zeros(cam.width * cam.height, np.int32),
                viewspace_points=np.zeros((n, 4), np.float32))
