"""fastgs_core_b200: the FastGS differentiable tile rasterizer on B200 (sm_100a).

Drop-in for the reference module ``fastgs_core`` (same primitive functions,
argument names, dict schemas and errors); kernels are in libfastgs_b200.so
(C ABI: include/fastgs_b200.h).
"""
from .api import (  # noqa: F401
    binning_forward,
    l1_dssim_loss,
    preprocess_backward,
    preprocess_forward,
    rasterize_backward,
    rasterize_forward,
    rasterize_gaussians,
    rasterize_gaussians_forward,
    sort_key_bits,
    sort_keys,
    sort_status,
    tile_grid,
    tile_prep_forward,
)

__version__ = "0.1.0"
