"""ctypes binding of libfastgs_b200.so (the C ABI declared in include/fastgs_b200.h).

There is no fallback: if the library is missing or fails to load, every call
raises. Status codes map to the exception types the reference's nanobind layer
raises (std::invalid_argument -> ValueError, std::runtime_error -> RuntimeError).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfastgs_b200.so")

FGS_OK, FGS_ERR_INVALID, FGS_ERR_CUDA, FGS_ERR_TIMEOUT, FGS_ERR_CAPACITY = range(5)

_p = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f = C.c_float
_sz = C.c_size_t


class PreprocessParams(C.Structure):
    _fields_ = [("n", _i32), ("degree", _i32), ("max_sh_coeffs", _i32), ("scale_modifier", _f),
                ("mult", _f), ("tan_fovx", _f), ("tan_fovy", _f), ("image_width", _i32),
                ("image_height", _i32), ("use_cov3d_precomp", _i32), ("use_colors_precomp", _i32)]


class RasterParams(C.Structure):
    _fields_ = [("image_width", _i32), ("image_height", _i32), ("num_tiles", _i32),
                ("bucket_sum", _i64), ("num_gaussians", _i32), ("get_flag", _i32),
                ("tile_order", _p), ("contrib_mask", _p), ("sparse_samples", _i32)]


# name -> (restype, argtypes)
_SIGS = {
    "fgs_last_error": (C.c_char_p, []),
    "fgs_version": (C.c_int, []),
    "fgs_preprocess_forward": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 22),
    "fgs_scan_scratch_bytes": (_sz, [_i64]),
    "fgs_inclusive_scan_u32": (C.c_int, [_i64, _p, _p, _p, _p, _p]),
    "fgs_duplicate_with_keys": (C.c_int, [_i32, _f, _i32, _i32, _p, _p, _p, _p, _p, _i64, _p, _p, _p]),
    "fgs_sort_workspace_bytes": (_sz, [_i64, _i32]),
    "fgs_sort_pairs": (C.c_int, [_i64, _i32, _p, _p, _p, _p, _p, _sz, _p]),
    "fgs_sort_pairs_static": (C.c_int, [_i64, _i32, _p, _p, _p, _p, _p]),
    "fgs_sort_status": (C.c_int, [_p, _p]),
    "fgs_sort_set_test_hooks": (C.c_int, [_i32, _i32]),
    "fgs_tile_prep": (C.c_int, [_i64, _i32, _p, _p, _p, _p, _p, _p]),
    "fgs_tile_order": (C.c_int, [_i32, _p, _p, _p]),
    "fgs_gather_rows": (C.c_int, [_i64, _i64, _p, _i32, _p, _p, _p, _p]),
    "fgs_densify_masks": (C.c_int, [_i64, _p, _p, _p, _f, _f, _f, _f, _p, _p]),
    "fgs_prune_masks": (C.c_int, [_i64, _p, _p, _f, _f, _f, _p, _p]),
    "fgs_split_fixup": (C.c_int, [_i64, _i64, _i64, _p, _i32, _p, _p]),
    "fgs_opacity_cap": (C.c_int, [_i64, _f, _p, _p, _p, _p]),
    "fgs_tile_prep_ordered": (C.c_int, [_i64, _i32] + [_p] * 7 + [_i64, _p]),
    "fgs_sort_pairs_bits": (C.c_int, [_i64, _i32, _i32] + [_p] * 5 + [_sz, _p]),
    "fgs_depth_order_workspace_bytes": (_sz, [_i32]),
    "fgs_depth_order": (C.c_int, [_i32] + [_p] * 5 + [_sz, _p]),
    "fgs_duplicate_with_keys_ordered": (C.c_int, [_i32, _f, _i32, _i32] + [_p] * 6 + [_i64, _p, _p, _p]),
    "fgs_rasterize_forward": (C.c_int, [C.POINTER(RasterParams)] + [_p] * 18),
    "fgs_rasterize_backward": (C.c_int, [C.POINTER(RasterParams)] + [_p] * 20),
    "fgs_preprocess_backward": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 24),
    "fgs_activate_params": (C.c_int, [_i64, _p, _p, _p, _p, _p]),
    "fgs_preprocess_backward_train": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 11
                                      + [_i32, _p, _p, _p]),
    "fgs_preprocess_forward_train": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 15),
    "fgs_preprocess_forward_train_geometry": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 12),
    "fgs_preprocess_colors_train": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 6),
    "fgs_preprocess_backward_adam": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 14
                                     + [_f, _f, _f, _i32, _i32, _p, _p]),
    "fgs_loss_scratch_bytes": (_sz, [_i32, _i32]),
    "fgs_l1_dssim_loss": (C.c_int, [_i32, _i32, _p, _p, _f, _f, _p, _p, _p, _p]),
    "fgs_mse_loss": (C.c_int, [_i32, _i32, _p, _p, _f, _p, _p, _p, _p]),
    "fgs_adam_step": (C.c_int, [_i64, _p, _p, _p, _p, _i32, C.POINTER(_i64), C.POINTER(_f), _f, _f,
                                _f, _i32, _i32, _p]),
    "fgs_adam_step_multicast": (C.c_int, [_i64, _p, _p, _p, _p, _p, _i32, C.POINTER(_i64),
                                          C.POINTER(_f), _f, _f, _f, _i32, _i32, _p]),
    "fgs_adam_step_peers": (C.c_int, [_i64, _i32, _i32, C.POINTER(_p), C.POINTER(_p), _p, _p, _i32,
                                      C.POINTER(_i64), C.POINTER(_f), _f, _f, _f, _i32, _i32, _p]),
    "fgs_set_exchange_grid": (C.c_int, [_i32]),
    "fgs_adam_step_gathered": (C.c_int, [_i64, _i32, C.POINTER(_p), _p, _p, _p, _i32,
                                         C.POINTER(_i64), C.POINTER(_f), _f, _f, _f, _i32, _i32, _p]),
    "fgs_preprocess_backward_push": (C.c_int, [C.POINTER(PreprocessParams)] + [_p] * 11
                                     + [_i32, _i64, C.POINTER(_p), _p, _p]),
    "fgs_adam_step_owner": (C.c_int, [_i64, _i32, _i32, C.POINTER(_p), _p, _p, _p, _p, _i32,
                                      C.POINTER(_i64), C.POINTER(_f), _f, _f, _f, _i32, _i32, _p]),
    "fgs_metric_map": (C.c_int, [_i64, _p, _p, _f, _p, _p, _p, _p]),
    "fgs_score_accumulate": (C.c_int, [_i64, _p, _p, _i64, _p, _p, _p]),
    "fgs_score_finalize": (C.c_int, [_i64, _p, _p, _i32, _p, _p, _p, _p]),
}

_lib = None


def lib() -> C.CDLL:
    """Load the library (once). Raises if it is missing: there is no CPU path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} not found: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
                " or `python fastgs_core_b200/csrc/build.py` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, what: str) -> None:
    if status == FGS_OK:
        return
    msg = lib().fgs_last_error().decode(errors="replace")
    if status == FGS_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed (status {status}): {msg}")
