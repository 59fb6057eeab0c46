"""Host-side behaviour of the Python API that needs no GPU: the reference's
argument validation and error texts (fastgs_core/binding/binding.cpp)."""
import numpy as np
import pytest
import torch

import fastgs_core_b200 as fg


def _base(n=4):
    return dict(means3d=torch.zeros(n, 3), opacities=torch.ones(n), viewmat=torch.eye(4),
                projmat=torch.eye(4), cam_pos=torch.zeros(3), viewspace_points=torch.zeros(n, 4))


def test_preprocess_missing_key():
    d = _base()
    del d["cam_pos"]
    with pytest.raises(RuntimeError, match="preprocess_forward missing required input tensor: cam_pos"):
        fg.preprocess_forward(d, 16, 16)


def test_preprocess_color_path_exclusive():
    d = _base()
    d.update(colors_precomp=torch.ones(4, 3), dc=torch.zeros(4, 3), sh=torch.zeros(4, 0, 3),
             cov3d_precomp=torch.ones(4, 6))
    with pytest.raises(RuntimeError, match="exactly one color path"):
        fg.preprocess_forward(d, 16, 16)


def test_preprocess_geometry_path_exclusive():
    d = _base()
    d.update(colors_precomp=torch.ones(4, 3))
    with pytest.raises(RuntimeError, match="exactly one geometry path: either cov3d_precomp OR scales\\+quats"):
        fg.preprocess_forward(d, 16, 16)


def test_rasterize_gaussians_names():
    d = dict(means3d=torch.zeros(2, 3), background=torch.zeros(3), opacities=torch.ones(2),
             metric_map=torch.zeros(256, dtype=torch.int32), viewmatrix=torch.eye(4),
             projmatrix=torch.eye(4))
    with pytest.raises(RuntimeError, match="rasterize_gaussians_forward missing required input tensor: campos"):
        fg.rasterize_gaussians(d, 16, 16)
    d["campos"] = torch.zeros(3)
    d["colors"] = torch.ones(2, 3)
    with pytest.raises(RuntimeError, match="scales\\+rotations"):
        fg.rasterize_gaussians(d, 16, 16)


def test_block_size_rejected():
    with pytest.raises(ValueError, match="16"):
        fg.preprocess_forward(_base(), 16, 16, block_x=8, block_y=8)


def test_cpu_tensors_rejected():
    d = _base()
    d.update(colors_precomp=torch.ones(4, 3), cov3d_precomp=torch.ones(4, 6))
    with pytest.raises(ValueError, match="CUDA"):
        fg.preprocess_forward(d, 16, 16)


def test_rasterize_forward_shape_errors():
    with pytest.raises(ValueError, match=r"means2d with shape \(N, 2\)"):
        fg.rasterize_forward(None, None, None, torch.zeros(3, 3), None, None, None, None, None, None,
                             torch.zeros(3, 4), 16, 16, 16, 16, 3, 1, 0)
    with pytest.raises(ValueError, match="share the same N"):
        fg.rasterize_forward(None, None, None, torch.zeros(3, 2), None, None, None, None, None, None,
                             torch.zeros(2, 4), 16, 16, 16, 16, 3, 1, 0)


def test_helpers():
    assert fg.tile_grid(1920, 1080) == (120, 68)
    assert fg.sort_key_bits(8160) == 45
    assert fg.sort_key_bits(1) == 33


def test_alias_package():
    import fastgs_core
    from fastgs_core import _fastgs_core

    assert fastgs_core.rasterize_gaussians is fg.rasterize_gaussians
    assert _fastgs_core.preprocess_forward is fg.preprocess_forward
    assert np.isclose(1.0, 1.0)
