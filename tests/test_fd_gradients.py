"""Finite-difference check of the gradients on the reference's numeric-check
fixtures (scripts/backward_numeric_check.py:22-145): the one-splat raster
primitive (means2d), the end-to-end path (means3d, opacities,
colors_precomp), preprocess cov3D (scales, rotations) and preprocess SH at
degree 2 (dc, sh).

The analytic gradients restate the reference's backward kernels; this checks
that they are derivatives of the forward pass, which the bit-level parity
tests cannot. Central differences use the CPU oracle in libm mode (the
reference's arithmetic) with the reference's step 1e-3, formed in float64
from the float32 losses. Every entry of each gradient is checked, not one
sample. Tolerance: 2e-2 relative to the largest entry of the gradient (the
reference's own script accepts 0.5). The CPU test checks the oracle's
backward; the GPU test checks the CUDA kernels through the public API.

One convention shows up here and is the reference's: the raster VJP returns
the means2d gradient in NDC units, i.e. the pixel-space derivative times
(W/2, H/2) (fastgs_rasterize_backward.metal:101-102 applies the factor there
and the projection Jacobian of fastgs_preprocess_backward.metal:188-205
leaves it out), so the end-to-end gradients are true derivatives. The
means2d check divides by that factor, at the reference's point (8, 8), where
symmetry makes the gradient zero, and at an off-centre point.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle

EPS = 1e-3
TOL = 2e-2


def _err(a, b):
    """Max error relative to the largest entry (floor 1e-3: a gradient that
    is zero by symmetry is compared against the step's noise)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-3))


# ------------------------------------------------------------- fixtures
def raster_inputs(means2d):
    return dict(ranges=np.array([[0, 1]], np.uint32), point_list=np.array([0], np.uint32),
                bucket_offsets=np.array([1], np.uint32),
                means2d=np.asarray(means2d, np.float32).reshape(1, 2),
                colors=np.array([[1.0, 1.0, 1.0]], np.float32),
                conic_opacity=np.array([[1.0, 0.0, 1.0, 0.5]], np.float32),
                background=np.zeros(3, np.float32), metric_map=np.zeros(256, np.int32))


def raster_loss(o, means2d, grad=False):
    a = raster_inputs(means2d)
    a.update(bucket_to_tile=np.zeros(256, np.uint32), sampled_t=np.zeros(256, np.float32),
             sampled_ar=np.zeros(3 * 256 + 96, np.float32), final_t=np.zeros(256, np.float32),
             n_contrib=np.zeros(256, np.uint32), max_contrib=np.zeros(1, np.uint32),
             pixel_colors=np.zeros((3, 256), np.float32), out_color=np.zeros((3, 256), np.float32),
             metric_count=np.zeros(0, np.int32), metric_count_buf=np.zeros(1, np.int32))
    o.render_forward(16, 16, 1, 1, 0, a)
    if not grad:
        return float(a["out_color"].astype(np.float64).sum())
    g = dict(dL_dout=np.ones((3, 256), np.float32), dmeans2d=np.zeros((1, 2), np.float32),
             dcolors=np.zeros((1, 3), np.float32), dconic=np.zeros((1, 4), np.float32),
             dviewspace=np.zeros((1, 4), np.float32))
    o.render_backward(16, 16, 1, 1, a, g)
    return g["dmeans2d"]


N = 8


def e2e_inputs(means3d=None, opacities=None, colors=None):
    base = dict(background=np.zeros(3, np.float32),
                means3d=np.array([[0.1, 0.1, 1.2 + 0.01 * i] for i in range(N)], np.float32),
                colors_precomp=np.array([[1.0, 0.6, 0.2]] * N, np.float32),
                opacities=np.full(N, 0.6, np.float32),
                cov3d_precomp=np.array([[1.0, 0.0, 0.0, 1.0, 0.0, 1.0]] * N, np.float32),
                metric_map=np.zeros(32 * 32, np.int32), viewmatrix=np.eye(4, dtype=np.float32),
                projmatrix=np.eye(4, dtype=np.float32), campos=np.zeros(3, np.float32),
                viewspace_points=np.zeros((N, 4), np.float32))
    if means3d is not None:
        base["means3d"] = np.asarray(means3d, np.float32)
    if opacities is not None:
        base["opacities"] = np.asarray(opacities, np.float32)
    if colors is not None:
        base["colors_precomp"] = np.asarray(colors, np.float32)
    return base


def e2e_loss(o, ins, grad=False):
    f = o.forward(ins, W=32, H=32, tan_fovx=1.0, tan_fovy=1.0, degree=0)
    if not grad:
        return float(f["out_color"].astype(np.float64).sum())
    return o.backward(f, np.ones((3, 32 * 32), np.float32))


def pre_inputs(kind, x):
    ins = dict(means3d=np.array([[0.1, 0.1, 1.2 + 0.01 * i] for i in range(N)], np.float32),
               opacities=np.full(N, 0.6, np.float32), viewmatrix=np.eye(4, dtype=np.float32),
               projmatrix=np.eye(4, dtype=np.float32), campos=np.zeros(3, np.float32),
               viewspace_points=np.zeros((N, 4), np.float32), background=np.zeros(3, np.float32))
    if kind == "cov":
        ins.update(colors_precomp=np.array([[1.0, 0.6, 0.2]] * N, np.float32),
                   scales=np.asarray(x[0], np.float32), rotations=np.asarray(x[1], np.float32))
    else:
        ins.update(cov3d_precomp=np.array([[1.0, 0.0, 0.0, 1.0, 0.0, 1.0]] * N, np.float32),
                   dc=np.asarray(x[0], np.float32), sh=np.asarray(x[1], np.float32))
    return ins


def pre_loss(o, kind, x, grad=False):
    """sum(cov3d) (kind "cov") or sum(rgb) at degree 2 (kind "sh") of
    preprocess_forward on a 16x16 image, and its gradient."""
    ins = pre_inputs(kind, x)
    deg = 0 if kind == "cov" else 2
    f = o.forward(ins, W=16, H=16, tan_fovx=1.0, tan_fovy=1.0, degree=deg)
    key = "cov3d" if kind == "cov" else "rgb"
    if not grad:
        return float(f[key].astype(np.float64).sum())
    # the preprocess VJP for a cotangent of ones on that output alone
    n = N
    pg = dict(dcov3d=np.zeros((n, 6), np.float32), drgb=np.zeros((n, 3), np.float32),
              dxys=np.zeros((n, 2), np.float32), dconic=np.zeros((n, 4), np.float32),
              dvs=np.zeros((n, 4), np.float32), ddepths=np.zeros(n, np.float32),
              dmeans3d=np.zeros((n, 3), np.float32), ddc=np.zeros((n, 3), np.float32),
              dsh=np.zeros_like(f["_ins"]["sh"]), dcolors_precomp=np.zeros((n, 3), np.float32),
              dopacities=np.zeros(n, np.float32), dscales=np.zeros((n, 3), np.float32),
              dquats=np.zeros((n, 4), np.float32), dvs_in=np.zeros((n, 4), np.float32))
    pg["dcov3d" if kind == "cov" else "drgb"][:] = 1.0
    p = f["_params"]
    o.preprocess_backward(n, 16, 16, p["use_cov"], p["use_col"], p["scale_modifier"], p["tan_fovx"],
                          p["tan_fovy"], p["degree"], p["maxc"],
                          dict(ins=f["_ins"], cov3d=f["cov3d"], radii=f["radii"], clamped=f["clamped"]),
                          pg)
    return pg


def central(fn, x):
    x = np.asarray(x, np.float32)
    g = np.zeros(x.shape, np.float64)
    for idx in np.ndindex(x.shape):
        xp, xm = x.copy(), x.copy()
        xp[idx] += EPS
        xm[idx] -= EPS
        g[idx] = (fn(xp) - fn(xm)) / (2.0 * EPS)
    return g


SCALES = np.array([[1.0, 1.1, 1.2]] * N, np.float32)
QUATS = np.array([[1.0, 0.0, 0.0, 0.0]] * N, np.float32)
DC = np.array([[0.5, 0.4, 0.3]] * N, np.float32)
SH = np.array([[[0.1, 0.2, 0.3], [0.0, 0.0, 0.0], [0.0, 0.0, 0.0], [0.05, -0.02, 0.01],
                [0.0, 0.0, 0.0], [0.0, 0.0, 0.0], [0.0, 0.0, 0.0], [0.0, 0.0, 0.0]]] * N, np.float32)
M3D = np.array([[0.1, 0.1, 1.2 + 0.01 * i] for i in range(N)], np.float32)
OPA = np.full(N, 0.6, np.float32)
COL = np.array([[1.0, 0.6, 0.2]] * N, np.float32)


M2D = (np.array([[8.0, 8.0]], np.float32), np.array([[8.3, 7.6]], np.float32))
NDC = np.array([[8.0, 8.0]])  # (W/2, H/2) of the 16x16 raster fixture


def numeric_grads():
    o = Oracle("libm")
    return {
        "means2d": central(lambda z: raster_loss(o, z), M2D[0]),
        "means2d_off": central(lambda z: raster_loss(o, z), M2D[1]),
        "means3d": central(lambda m: e2e_loss(o, e2e_inputs(means3d=m)), M3D),
        "opacities": central(lambda a: e2e_loss(o, e2e_inputs(opacities=a)), OPA),
        "colors_precomp": central(lambda c: e2e_loss(o, e2e_inputs(colors=c)), COL),
        "scales": central(lambda s: pre_loss(o, "cov", (s, QUATS)), SCALES),
        "rotations": central(lambda q: pre_loss(o, "cov", (SCALES, q)), QUATS),
        "dc": central(lambda d: pre_loss(o, "sh", (d, SH)), DC),
        "sh": central(lambda s: pre_loss(o, "sh", (DC, s)), SH),
    }


_NUM = {}


def num(k):
    if not _NUM:
        _NUM.update(numeric_grads())
    return _NUM[k]


def test_oracle_backward_is_the_derivative():
    o = Oracle("libm")
    b = e2e_loss(o, e2e_inputs(), grad=True)
    cov = pre_loss(o, "cov", (SCALES, QUATS), grad=True)
    sh = pre_loss(o, "sh", (DC, SH), grad=True)
    ana = {"means2d": raster_loss(o, M2D[0], grad=True) / NDC,
           "means2d_off": raster_loss(o, M2D[1], grad=True) / NDC,
           "means3d": b["dmeans3d"], "opacities": b["dopacities"], "colors_precomp": b["dcolors_precomp"],
           "scales": cov["dscales"], "rotations": cov["dquats"], "dc": sh["ddc"], "sh": sh["dsh"]}
    for k, a in ana.items():
        n = num(k)
        assert _err(a.reshape(n.shape), n) < TOL, (k, _err(a.reshape(n.shape), n))


@pytest.mark.gpu
def test_gpu_gradients_are_the_derivative(cuda_dev):
    import torch

    import fastgs_core_b200 as fg

    def t(x, grad=True):
        return torch.from_numpy(np.ascontiguousarray(x)).to(cuda_dev).requires_grad_(grad)

    # raster primitive (rasterize_forward + its VJP, NDC units)
    got = {}
    for key, pt in (("means2d", M2D[0]), ("means2d_off", M2D[1])):
        a = raster_inputs(pt)
        m2 = t(a["means2d"])
        out = fg.rasterize_forward(t(a["ranges"], False), t(a["point_list"], False),
                                   t(a["bucket_offsets"], False), m2, t(a["colors"], False),
                                   t(a["conic_opacity"], False), t(a["background"], False),
                                   torch.ones(1, dtype=torch.int32, device=cuda_dev),
                                   t(a["metric_map"], False),
                                   torch.zeros(1, dtype=torch.int32, device=cuda_dev),
                                   torch.zeros((1, 4), device=cuda_dev), 16, 16, 16, 16, 3, 1, 1, False)
        out["out_color"].sum().backward()
        got[key] = m2.grad.cpu().numpy() / NDC
    # end-to-end
    ins = {k: t(v, k in ("means3d", "opacities", "colors_precomp") and v.dtype == np.float32)
           for k, v in e2e_inputs().items()}
    fg.rasterize_gaussians(ins, 32, 32, 16, 16, 1.0, 1.0, 0)["out_color"].sum().backward()
    for k in ("means3d", "opacities", "colors_precomp"):
        got[k] = ins[k].grad.cpu().numpy()
    # preprocess cov3D and SH (degree 2)
    for kind, x, names, key in (("cov", (SCALES, QUATS), ("scales", "rotations"), "cov3d"),
                                ("sh", (DC, SH), ("dc", "sh"), "rgb")):
        p = pre_inputs(kind, x)
        d = {k: t(v, k in names) for k, v in p.items() if k not in ("background",)}
        d = {("viewmat" if k == "viewmatrix" else "projmat" if k == "projmatrix" else
              "cam_pos" if k == "campos" else "quats" if k == "rotations" else k): v for k, v in d.items()}
        outp = fg.preprocess_forward(d, 16, 16, degree=0 if kind == "cov" else 2)
        outp[key].sum().backward()
        got[names[0]] = d[names[0]].grad.cpu().numpy()
        got[names[1]] = d["quats" if names[1] == "rotations" else names[1]].grad.cpu().numpy()
    for k, g in got.items():
        n = num(k)
        assert _err(g.reshape(n.shape), n) < TOL, (k, _err(g.reshape(n.shape), n))
