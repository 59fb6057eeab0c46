"""Shared helpers for the GPU parity tests (test infrastructure)."""
import numpy as np
import torch

import fastgs_core_b200 as fg

INT_KEYS = ("radii", "point_offsets", "point_list_keys", "point_list", "ranges", "bucket_count",
            "bucket_offsets")
GEOM = {"geom_means2d": "xys", "geom_depths": "depths", "geom_cov3d": "cov3d", "geom_rgb": "rgb",
        "geom_conic_opacity": "conic_opacity", "geom_tiles_touched": "tiles_touched",
        "geom_clamped": "clamped", "viewspace_points": "viewspace_points",
        "img_final_t": "final_t", "img_n_contrib": "n_contrib", "img_max_contrib": "max_contrib",
        "img_pixel_colors": "pixel_colors", "sample_t": "sampled_t", "sample_ar": "sampled_ar"}
LEAVES = ("means3d", "dc", "sh", "colors_precomp", "opacities", "scales", "rotations",
          "cov3d_precomp", "viewspace_points")
GRAD_MAP = {"means3d": "dmeans3d", "dc": "ddc", "sh": "dsh", "colors_precomp": "dcolors_precomp",
            "opacities": "dopacities", "scales": "dscales", "rotations": "dquats",
            "viewspace_points": "dviewspace_points"}


def to_dev(ins_np, dev, grad=True):
    out = {}
    for k, v in ins_np.items():
        t = torch.from_numpy(np.ascontiguousarray(v)).to(dev)
        if grad and k in LEAVES and t.dtype == torch.float32:
            t.requires_grad_(True)
        out[k] = t
    return out


def run_chain(ins_np, W, H, tanx, tany, degree, dev, cot=None, get_flag=False):
    ins = to_dev(ins_np, dev)
    out = fg.rasterize_gaussians(ins, W, H, 16, 16, tanx, tany, degree, 1.0, 1.0, False, get_flag)
    grads = {}
    if cot is not None and out["out_color"].numel():
        out["out_color"].backward(torch.from_numpy(cot).to(dev))
        grads = {k: ins[k].grad.detach().cpu().numpy() for k in LEAVES
                 if k in ins and ins[k].grad is not None}
    res = {}
    for k, v in out.items():
        res[k] = v.detach().cpu().numpy() if torch.is_tensor(v) else v
    return res, grads


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-12)) if b.size else 0.0
