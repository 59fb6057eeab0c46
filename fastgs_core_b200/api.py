"""Python-facing primitive API, mirroring the reference module ``fastgs_core``.

Functions, argument names, defaults, dict keys and error texts follow the
reference's nanobind module (fastgs_core/binding/binding.cpp:512-610):
``preprocess_forward``, ``binning_forward``, ``tile_prep_forward``,
``rasterize_forward``, ``rasterize_gaussians`` / ``rasterize_gaussians_forward``.
Tensors are torch CUDA tensors instead of MLX arrays. Gradients flow through
torch autograd exactly where they flow through MLX autodiff in the reference:
``preprocess_forward`` and ``rasterize_forward`` are differentiable primitives
(their VJPs are FastGSPreprocess::vjp, fastgs_core/fastgs_preprocess.cpp:191-206,
and FastGSRasterize::vjp, fastgs_core/fastgs_rasterize.cpp:191-206), binning and
tile prep are not. New here: the VJPs are also callable directly
(``preprocess_backward``, ``rasterize_backward``), and the sort the reference
hides inside ``rasterize_gaussians`` is exposed as ``sort_keys``.

Every kernel runs through libfastgs_b200.so on the current CUDA stream; there
is no CPU path (CPU tensors are rejected).
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import _lib
from ._lib import PreprocessParams, RasterParams, check, lib

BLOCK = 16

__all__ = [
    "preprocess_forward", "binning_forward", "sort_keys", "tile_prep_forward", "rasterize_forward",
    "rasterize_gaussians", "rasterize_gaussians_forward", "preprocess_backward",
    "rasterize_backward", "tile_grid", "sort_key_bits", "sort_status", "l1_dssim_loss",
]


# ------------------------------------------------------------------ helpers
def _p(t: torch.Tensor | None):
    if t is None or t.numel() == 0:
        return None
    return C.c_void_p(t.data_ptr())


def _stream(dev: torch.device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _f32(t, dev=None) -> torch.Tensor:
    t = torch.as_tensor(t)
    if dev is not None and t.device != dev:
        t = t.to(dev)
    if not t.is_cuda:
        raise ValueError("fastgs_core_b200 runs on CUDA tensors only (no CPU path)")
    return _aligned(t.detach().to(torch.float32).contiguous())


def _int_t(t, dtype, dev) -> torch.Tensor:
    t = torch.as_tensor(t)
    if t.device != dev:
        t = t.to(dev)
    if t.dtype != dtype:
        t = t.to(dtype)
    return _aligned(t.contiguous())


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The kernels read several inputs as 8- and 16-byte vectors; a view that
    starts inside an allocation is copied to a fresh (aligned) one."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def tile_grid(width: int, height: int) -> tuple[int, int]:
    return (width + BLOCK - 1) // BLOCK, (height + BLOCK - 1) // BLOCK


def sort_key_bits(num_tiles: int) -> int:
    """32 depth bits plus the bits needed for tile ids 0..num_tiles-1."""
    return 32 + max(1, int(max(num_tiles, 1) - 1).bit_length())


def _check_block(block_x: int, block_y: int) -> None:
    if block_x != BLOCK or block_y != BLOCK:
        raise ValueError(f"block_x/block_y must be {BLOCK} (the kernels use 16x16 tiles), "
                         f"got {block_x}x{block_y}")


class _Workspace:
    """Grow-only per-device scratch for the scan and the sort."""

    def __init__(self):
        self._bufs: dict[tuple, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, dev: torch.device, tag: str, nbytes: int) -> torch.Tensor:
        key = (dev.index, tag)
        with self._lock:
            b = self._bufs.get(key)
            if b is None or b.numel() < nbytes:
                b = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
                self._bufs[key] = b
            return b

    def peek(self, dev: torch.device, tag: str) -> torch.Tensor | None:
        with self._lock:
            return self._bufs.get((dev.index, tag))


_WS = _Workspace()


# ------------------------------------------------------------- preprocess
_PRE_OUT = ("radii", "xys", "depths", "cov3d", "rgb", "conic_opacity", "tiles_touched", "clamped",
            "viewspace_points")


def _pre_params(n, degree, maxc, scale_modifier, mult, tan_fovx, tan_fovy, W, H, use_cov, use_col):
    return PreprocessParams(n, degree, maxc, scale_modifier, mult, tan_fovx, tan_fovy, W, H,
                            int(use_cov), int(use_col))


def _run_preprocess(prm: PreprocessParams, t: dict, dev) -> dict:
    n = prm.n
    o = dict(
        radii=torch.empty(n, dtype=torch.int32, device=dev),
        xys=torch.empty((n, 2), dtype=torch.float32, device=dev),
        depths=torch.empty(n, dtype=torch.float32, device=dev),
        cov3d=torch.empty((n, 6), dtype=torch.float32, device=dev),
        rgb=torch.empty((n, 3), dtype=torch.float32, device=dev),
        conic_opacity=torch.empty((n, 4), dtype=torch.float32, device=dev),
        tiles_touched=torch.empty(n, dtype=torch.uint32, device=dev),
        clamped=torch.empty((n, 3), dtype=torch.bool, device=dev),
        viewspace_points=torch.empty((n, 4), dtype=torch.float32, device=dev),
    )
    st = lib().fgs_preprocess_forward(
        C.byref(prm), *[_p(t[k]) for k in ("means3d", "dc", "sh", "colors_precomp", "opacities",
                                           "scales", "quats", "cov3d_precomp", "viewmat", "projmat",
                                           "cam_pos", "viewspace_points")],
        *[_p(o[k]) for k in _PRE_OUT], _stream(dev))
    check(st, "preprocess_forward")
    return o


def _run_preprocess_backward(prm: PreprocessParams, t: dict, fwd: dict, cot: dict, dev) -> dict:
    n = prm.n
    z = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)  # noqa: E731
    e = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)  # noqa: E731
    maxc = prm.max_sh_coeffs
    g = dict(dmeans3d=e(n, 3), ddc=e(n, 3), dsh=e(n, maxc, 3), dcolors_precomp=e(n, 3),
             dopacities=e(n), dscales=e(n, 3), dquats=e(n, 4), dviewspace=e(n, 4))

    def c(k, *shape):
        v = cot.get(k)
        return z(*shape) if v is None else _f32(v, dev)

    # the cotangents are bound to names for the whole call: a raw pointer into
    # a temporary would dangle once the temporary is freed, and the caching
    # allocator would hand its memory to the next temporary
    dcov = cot.get("cov3d")
    dcov = None if dcov is None else _f32(dcov, dev)
    drgb, dxys = c("rgb", n, 3), c("xys", n, 2)
    dconic, dvs = c("conic_opacity", n, 4), c("viewspace_points", n, 4)
    st = lib().fgs_preprocess_backward(
        C.byref(prm), *[_p(t[k]) for k in ("means3d", "scales", "quats", "viewmat", "projmat",
                                           "cam_pos", "sh", "cov3d_precomp")],
        _p(fwd["cov3d"]), _p(dcov), _p(drgb), _p(dxys), _p(dconic), _p(dvs),
        _p(fwd["radii"]), _p(fwd["clamped"]),
        *[_p(g[k]) for k in ("dmeans3d", "ddc", "dsh", "dcolors_precomp", "dopacities", "dscales",
                             "dquats", "dviewspace")], _stream(dev))
    check(st, "preprocess_backward")
    return g


class _PreprocessFn(torch.autograd.Function):
    """FastGSPreprocess as a torch autograd node (VJP: fastgs_preprocess_backward)."""

    @staticmethod
    def forward(ctx, prm, tensors, means3d, dc, sh, colors_precomp, opacities, scales, quats,
                cov3d_precomp, viewspace_points):
        dev = means3d.device
        o = _run_preprocess(prm, tensors, dev)
        ctx.set_materialize_grads(False)  # unused outputs' cotangents stay None (no zero fills)
        ctx.prm = prm
        ctx.tensors = tensors
        ctx.fwd = {k: o[k] for k in ("cov3d", "radii", "clamped")}
        ctx.mark_non_differentiable(o["radii"], o["tiles_touched"], o["clamped"])
        return tuple(o[k] for k in _PRE_OUT)

    @staticmethod
    def backward(ctx, g_radii, g_xys, g_depths, g_cov3d, g_rgb, g_conic, g_tiles, g_clamped, g_vs):
        dev = ctx.tensors["means3d"].device
        cot = dict(xys=g_xys, cov3d=g_cov3d, rgb=g_rgb, conic_opacity=g_conic, viewspace_points=g_vs)
        g = _run_preprocess_backward(ctx.prm, ctx.tensors, ctx.fwd, cot, dev)
        zero = lambda t: None if t is None else torch.zeros_like(t)  # noqa: E731
        t = ctx.tensors
        return (None, None, g["dmeans3d"], g["ddc"] if t["dc"] is not None else None,
                g["dsh"] if t["sh"] is not None else None,
                g["dcolors_precomp"] if t["colors_precomp"] is not None else None,
                g["dopacities"].view_as(t["opacities"]),
                g["dscales"] if t["scales"] is not None else None,
                g["dquats"] if t["quats"] is not None else None,
                zero(t["cov3d_precomp"]),  # never written by the reference kernel
                g["dviewspace"])


def _prep_inputs(inputs: dict, names: dict, fn: str, dev=None):
    """Key lookup + the exclusive colour / geometry path rules of
    binding.cpp:424-453 (preprocess_forward) / :46-104 (rasterize_gaussians)."""

    def require(key):
        if key not in inputs:
            raise RuntimeError(f"{fn} missing required input tensor: {key}")
        return inputs[key]

    means3d = require("means3d")
    dev = dev or torch.as_tensor(means3d).device
    out = {"means3d": means3d, "opacities": require("opacities"),
           "viewmat": require(names["viewmat"]), "projmat": require(names["projmat"]),
           "cam_pos": require(names["cam_pos"])}
    cp = inputs.get("colors_precomp")
    if (cp is None or torch.as_tensor(cp).numel() == 0) and "colors" in names.get("aliases", ()):
        cp = inputs.get("colors")
    has_cp = cp is not None and torch.as_tensor(cp).numel() != 0
    has_sh = "dc" in inputs and "sh" in inputs
    if has_cp == has_sh:
        extra = " (or colors)" if "colors" in names.get("aliases", ()) else ""
        raise RuntimeError(f"{fn} expects exactly one color path: "
                           f"either colors_precomp{extra} OR dc+sh")
    cov = inputs.get("cov3d_precomp")
    has_cov = cov is not None and torch.as_tensor(cov).numel() != 0
    qkey = names["quats"]
    sc, q = inputs.get("scales"), inputs.get(qkey)
    has_sr = (sc is not None and torch.as_tensor(sc).numel() != 0 and q is not None
              and torch.as_tensor(q).numel() != 0)
    if has_cov == has_sr:
        raise RuntimeError(f"{fn} expects exactly one geometry path: "
                           f"either cov3d_precomp OR scales+{qkey}")
    out.update(colors_precomp=cp if has_cp else None, dc=inputs.get("dc") if has_sh else None,
               sh=inputs.get("sh") if has_sh else None, cov3d_precomp=cov if has_cov else None,
               scales=sc if has_sr else None, quats=q if has_sr else None)
    return out, has_cp, has_cov, dev


def _preprocess_apply(raw: dict, W, H, tan_fovx, tan_fovy, degree, scale_modifier, mult, use_col,
                      use_cov, vs, dev):
    means3d = raw["means3d"]
    n = int(means3d.shape[0])
    sh = raw["sh"]
    maxc = int(sh.shape[1]) if (sh is not None and torch.as_tensor(sh).dim() >= 2) else 0
    if not use_col and degree > 0 and maxc > 0 and (degree + 1) ** 2 - 1 > maxc:
        raise ValueError(f"degree {degree} needs {(degree + 1) ** 2 - 1} SH coefficients, sh has {maxc}")
    prm = _pre_params(n, int(degree), maxc, float(scale_modifier), float(mult), float(tan_fovx),
                      float(tan_fovy), int(W), int(H), use_cov, use_col)
    diff = {k: raw[k] for k in ("means3d", "dc", "sh", "colors_precomp", "opacities", "scales",
                                "quats", "cov3d_precomp")}
    diff["viewspace_points"] = vs
    det = {k: (None if v is None else _f32(v, dev)) for k, v in diff.items()}
    det["opacities"] = det["opacities"].reshape(-1)
    for k in ("viewmat", "projmat", "cam_pos"):
        det[k] = _f32(raw[k], dev).reshape(-1)
    if det["means3d"].shape != (n, 3):
        raise ValueError("means3d must have shape (N, 3)")
    if det["viewspace_points"].shape != (n, 4):
        raise ValueError("viewspace_points must have shape (N, 4)")
    args = [torch.as_tensor(diff[k]) if diff[k] is not None else None
            for k in ("means3d", "dc", "sh", "colors_precomp", "opacities", "scales", "quats",
                      "cov3d_precomp", "viewspace_points")]
    outs = _PreprocessFn.apply(prm, det, *args)
    return dict(zip(_PRE_OUT, outs)), prm


def preprocess_forward(inputs: dict, image_width: int, image_height: int, block_x: int = 16,
                       block_y: int = 16, tan_fovx: float = 1.0, tan_fovy: float = 1.0,
                       degree: int = 0, scale_modifier: float = 1.0, mult: float = 1.0,
                       prefiltered: bool = False) -> dict:
    """binding.cpp:397-508. Required keys: means3d, opacities, viewmat, projmat,
    cam_pos, viewspace_points; exactly one of colors_precomp / dc+sh and one of
    cov3d_precomp / scales+quats. Returns radii, xys, depths, cov3d, rgb,
    conic_opacity, tiles_touched, clamped, viewspace_points."""
    _check_block(block_x, block_y)
    names = dict(viewmat="viewmat", projmat="projmat", cam_pos="cam_pos", quats="quats")
    if "viewspace_points" not in inputs:
        raise RuntimeError("preprocess_forward missing required input tensor: viewspace_points")
    raw, use_col, use_cov, dev = _prep_inputs(inputs, names, "preprocess_forward")
    out, _ = _preprocess_apply(raw, image_width, image_height, tan_fovx, tan_fovy, degree,
                               scale_modifier, mult, use_col, use_cov, inputs["viewspace_points"], dev)
    return out


def preprocess_backward(inputs: dict, forward_outputs: dict, cotangents: dict, image_width: int,
                        image_height: int, tan_fovx: float = 1.0, tan_fovy: float = 1.0,
                        degree: int = 0, scale_modifier: float = 1.0) -> dict:
    """VJP of preprocess_forward (fastgs_core/fastgs_preprocess_backward.cpp:39-183).
    ``cotangents`` may hold xys, cov3d, rgb, conic_opacity, viewspace_points.
    Returns d_means3d, d_dc, d_sh, d_colors_precomp, d_opacities, d_scales,
    d_quats, d_viewspace_points (rows of culled Gaussians are zero)."""
    names = dict(viewmat="viewmat", projmat="projmat", cam_pos="cam_pos", quats="quats")
    raw, use_col, use_cov, dev = _prep_inputs(inputs, names, "preprocess_backward")
    n = int(raw["means3d"].shape[0])
    sh = raw["sh"]
    maxc = int(sh.shape[1]) if (sh is not None and torch.as_tensor(sh).dim() >= 2) else 0
    prm = _pre_params(n, int(degree), maxc, float(scale_modifier), 1.0, float(tan_fovx),
                      float(tan_fovy), int(image_width), int(image_height), use_cov, use_col)
    t = {k: (None if raw[k] is None else _f32(raw[k], dev)) for k in (
        "means3d", "dc", "sh", "colors_precomp", "opacities", "scales", "quats", "cov3d_precomp")}
    for k in ("viewmat", "projmat", "cam_pos"):
        t[k] = _f32(raw[k], dev).reshape(-1)
    fwd = dict(cov3d=_f32(forward_outputs["cov3d"], dev),
               radii=_int_t(forward_outputs["radii"], torch.int32, dev),
               clamped=_int_t(forward_outputs["clamped"], torch.bool, dev))
    g = _run_preprocess_backward(prm, t, fwd, cotangents, dev)
    return dict(d_means3d=g["dmeans3d"], d_dc=g["ddc"], d_sh=g["dsh"],
                d_colors_precomp=g["dcolors_precomp"], d_opacities=g["dopacities"],
                d_scales=g["dscales"], d_quats=g["dquats"], d_viewspace_points=g["dviewspace"])


# ---------------------------------------------------------------- binning
def _scan(tiles_touched: torch.Tensor, dev) -> tuple[torch.Tensor, torch.Tensor]:
    n = tiles_touched.numel()
    out = torch.empty(n, dtype=torch.uint32, device=dev)
    total = torch.empty(1, dtype=torch.uint64, device=dev)
    scratch = _WS.get(dev, "scan", int(lib().fgs_scan_scratch_bytes(n)))
    check(lib().fgs_inclusive_scan_u32(n, _p(tiles_touched), _p(out), _p(total), _p(scratch),
                                       _stream(dev)), "inclusive_scan")
    return out, total


def binning_forward(xys, depths, point_offsets, conic_opacity, tiles_touched, mult: float,
                    tile_bounds_x: int, tile_bounds_y: int, tile_bounds_z: int,
                    num_rendered: int) -> dict:
    """binding.cpp:345-375 (FastGSBinning). num_rendered == 0 gives empty outputs."""
    dev = torch.as_tensor(xys).device
    num_rendered = int(num_rendered)
    keys = torch.empty(num_rendered, dtype=torch.uint64, device=dev)
    vals = torch.empty(num_rendered, dtype=torch.uint32, device=dev)
    if num_rendered > 0:
        # converted inputs stay bound to names until the call returns (a raw
        # pointer into a freed temporary could be handed to the next one)
        xys = _f32(xys, dev)
        depths = _f32(depths, dev)
        offs = _int_t(point_offsets, torch.uint32, dev)
        conic = _f32(conic_opacity, dev)
        tiles = _int_t(tiles_touched, torch.uint32, dev)
        n = xys.shape[0]
        check(lib().fgs_duplicate_with_keys(
            n, float(mult), int(tile_bounds_x), int(tile_bounds_y), _p(xys), _p(depths), _p(offs),
            _p(conic), _p(tiles), num_rendered, _p(keys), _p(vals), _stream(dev)), "binning_forward")
    return {"point_list_keys_unsorted": keys, "point_list_unsorted": vals}


def sort_keys(keys: torch.Tensor, values: torch.Tensor, num_tiles: int | None = None,
              key_bits: int | None = None, check_status: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Stable ascending sort of uint64 keys with their uint32 values (the
    mx::argsort + take of binding.cpp:195-197) by the onesweep radix sort.
    check_status synchronises and raises RuntimeError if a bounded look-back
    wait gave up (fgs_sort_status); without it the sort stays asynchronous
    and ``sort_status(keys.device)`` reports later."""
    dev = keys.device
    k = keys.numel()
    if key_bits is None:
        key_bits = 64 if num_tiles is None else sort_key_bits(int(num_tiles))
    ko = torch.empty_like(keys)
    vo = torch.empty_like(values)
    if k:
        nbytes = int(lib().fgs_sort_workspace_bytes(k, key_bits))
        ws = _WS.get(dev, "sort", nbytes)
        kin, vin = keys.contiguous(), values.contiguous()  # alive for the whole call
        check(lib().fgs_sort_pairs(k, int(key_bits), _p(kin), _p(vin), _p(ko), _p(vo), _p(ws),
                                   ws.numel(), _stream(dev)), "sort_keys")
        if check_status:
            sort_status(dev)
    return ko, vo


def sort_status(dev) -> None:
    """Synchronise and raise RuntimeError if the last sort_keys on ``dev``
    had a look-back wait give up (its output is then undefined)."""
    dev = torch.device(dev)
    ws = _WS.peek(dev, "sort")
    if ws is not None:  # no sort has run on dev otherwise
        check(lib().fgs_sort_status(_p(ws), _stream(dev)), "sort_keys")


def _tile_prep(keys, num_rendered, num_tiles, dev):
    ranges = torch.empty((num_tiles, 2), dtype=torch.uint32, device=dev)
    bucket_count = torch.empty(num_tiles, dtype=torch.uint32, device=dev)
    bucket_offsets = torch.empty(num_tiles, dtype=torch.uint32, device=dev)
    bucket_sum = torch.zeros(1, dtype=torch.uint64, device=dev)
    check(lib().fgs_tile_prep(int(num_rendered), int(num_tiles), _p(keys), _p(ranges),
                              _p(bucket_count), _p(bucket_offsets), _p(bucket_sum), _stream(dev)),
          "tile_prep")
    return ranges, bucket_count, bucket_offsets, bucket_sum


def tile_prep_forward(point_list_keys, num_rendered: int, num_tiles: int) -> dict:
    """binding.cpp:377-395 (FastGSTilePrep): ranges [T,2] and bucket_count [T]."""
    dev = torch.as_tensor(point_list_keys).device
    if int(num_tiles) == 0:
        return {"ranges": torch.zeros((0, 2), dtype=torch.uint32, device=dev),
                "bucket_count": torch.zeros(0, dtype=torch.uint32, device=dev)}
    keys = _int_t(point_list_keys, torch.uint64, dev)
    ranges, bucket_count, _, _ = _tile_prep(keys, int(num_rendered), int(num_tiles), dev)
    return {"ranges": ranges, "bucket_count": bucket_count}


# -------------------------------------------------------------- rasterize
_RAS_OUT = ("bucket_to_tile", "sampled_t", "sampled_ar", "final_t", "n_contrib", "max_contrib",
            "pixel_colors", "out_color", "metric_count")


def _run_rasterize(rp: RasterParams, t: dict, dev) -> dict:
    P = rp.image_width * rp.image_height
    B = rp.bucket_sum
    o = dict(
        bucket_to_tile=torch.empty(B * 256, dtype=torch.uint32, device=dev),
        sampled_t=torch.empty(B * 256, dtype=torch.float32, device=dev),
        sampled_ar=torch.empty((3, B * 256), dtype=torch.float32, device=dev),
        final_t=torch.empty(P, dtype=torch.float32, device=dev),
        n_contrib=torch.empty(P, dtype=torch.uint32, device=dev),
        max_contrib=torch.empty(rp.num_tiles, dtype=torch.uint32, device=dev),
        pixel_colors=torch.empty((3, P), dtype=torch.float32, device=dev),
        out_color=torch.empty((3, P), dtype=torch.float32, device=dev),
    )
    mc = t["metric_count"]
    o["metric_count"] = (torch.empty_like(mc) if rp.get_flag else torch.zeros_like(mc))
    if "_tile_order" in t:
        # rasterize_gaussians: bucket arrays sized by a bound on the bucket
        # count, bucket_to_tile and the tile order written by tile prep; the
        # caller trims the outputs to the real count once it is known
        o["bucket_to_tile"] = t["_bucket_to_tile"]
        order = t["_tile_order"]
    else:
        # bucket_to_tile is declared [B*256] but only the first B entries are
        # written (fastgs_rasterize.metal:67-75); the rest stay at the zero fill
        if B:
            o["bucket_to_tile"][B:].zero_()
        # heaviest tiles first (same results in any order)
        order = torch.empty(rp.num_tiles, dtype=torch.uint32, device=dev)
        check(lib().fgs_tile_order(rp.num_tiles, _p(t["ranges"]), _p(order), _stream(dev)), "tile_order")
    rp.tile_order = order.data_ptr() if rp.num_tiles else None
    # per (bucket, pixel) contributing-splat bits: the backward pass of this
    # autograd node reads them instead of re-deciding every pair
    if B:
        o["contrib_mask"] = torch.empty(B * 256, dtype=torch.uint32, device=dev)
        rp.contrib_mask = o["contrib_mask"].data_ptr()
    st = lib().fgs_rasterize_forward(
        C.byref(rp), *[_p(t[k]) for k in ("ranges", "point_list", "bucket_offsets", "means2d",
                                          "colors", "conic_opacity", "background", "metric_map")],
        *[_p(o[k]) for k in _RAS_OUT], _stream(dev))
    check(st, "rasterize_forward")
    return o


def _run_rasterize_backward(rp: RasterParams, t: dict, o: dict, dout: torch.Tensor, dev) -> dict:
    n = t["means2d"].shape[0]
    # the kernel accumulates: one zeroed allocation, each part 16-byte aligned
    o1 = -(-2 * n // 4) * 4
    o2 = o1 + -(-3 * n // 4) * 4
    buf = torch.zeros(o2 + 8 * n, dtype=torch.float32, device=dev)
    g = dict(dmeans2d=buf[:2 * n].view(n, 2), dcolors=buf[o1:o1 + 3 * n].view(n, 3),
             dconic=buf[o2:o2 + 4 * n].view(n, 4), dviewspace=buf[o2 + 4 * n:].view(n, 4))
    st = lib().fgs_rasterize_backward(
        C.byref(rp), *[_p(t[k]) for k in ("ranges", "point_list", "bucket_offsets", "means2d",
                                          "colors", "conic_opacity", "background")],
        _p(dout), *[_p(o[k]) for k in ("bucket_to_tile", "sampled_t", "sampled_ar", "final_t",
                                       "n_contrib", "max_contrib", "pixel_colors")],
        *[_p(g[k]) for k in ("dmeans2d", "dcolors", "dconic", "dviewspace")], _stream(dev))
    check(st, "rasterize_backward")
    return g


class _RasterizeFn(torch.autograd.Function):
    """FastGSRasterize as a torch autograd node (VJP: fastgs_rasterize_backward);
    only the out_color cotangent is used, as fastgs_rasterize_backward.cpp:98."""

    @staticmethod
    def forward(ctx, rp, t, means2d, colors, conic_opacity, viewspace_points):
        dev = t["means2d"].device
        o = _run_rasterize(rp, t, dev)
        ctx.set_materialize_grads(False)  # only out_color's cotangent is used
        ctx.rp = rp
        ctx.t = t
        ctx.o = o
        outs = tuple(o[k] for k in _RAS_OUT)
        ctx.mark_non_differentiable(*[o[k] for k in _RAS_OUT if k != "out_color"])
        return outs

    @staticmethod
    def backward(ctx, *grads):
        g_out = grads[_RAS_OUT.index("out_color")]
        dev = ctx.t["means2d"].device
        if g_out is None:
            return None, None, None, None, None, None
        g = _run_rasterize_backward(ctx.rp, ctx.t, ctx.o, _f32(g_out, dev), dev)
        return None, None, g["dmeans2d"], g["dcolors"], g["dconic"], g["dviewspace"]


def _raster_tensors(ranges, point_list, per_tile_bucket_offset, means2d, colors, conic_opacity,
                    background, metric_map, metric_count, dev):
    return dict(ranges=_int_t(ranges, torch.uint32, dev), point_list=_int_t(point_list, torch.uint32, dev),
                bucket_offsets=_int_t(per_tile_bucket_offset, torch.uint32, dev),
                means2d=_f32(means2d, dev), colors=_f32(colors, dev),
                conic_opacity=_f32(conic_opacity, dev), background=_f32(background, dev).reshape(-1),
                metric_map=_int_t(metric_map, torch.int32, dev).reshape(-1),
                metric_count=_int_t(metric_count, torch.int32, dev))


def rasterize_forward(ranges, point_list, per_tile_bucket_offset, means2d, colors, conic_opacity,
                      background, radii, metric_map, metric_count, viewspace_points,
                      image_width: int, image_height: int, block_x: int, block_y: int,
                      num_channels: int, num_tiles: int, bucket_sum: int,
                      get_flag: bool = False) -> dict:
    """binding.cpp:286-343 (FastGSRasterize). Differentiable w.r.t. means2d,
    colors, conic_opacity and viewspace_points through out_color."""
    _check_block(block_x, block_y)
    if int(num_channels) != 3:
        raise ValueError("num_channels must be 3")
    m2 = torch.as_tensor(means2d)
    vs = torch.as_tensor(viewspace_points)
    if m2.dim() != 2 or m2.shape[1] != 2:
        raise ValueError("FastGSRasterize expects means2d with shape (N, 2).")
    if vs.dim() != 2 or vs.shape[1] != 4:
        raise ValueError("FastGSRasterize expects viewspace_points with shape (N, 4).")
    if m2.shape[0] != vs.shape[0]:
        raise ValueError("FastGSRasterize expects means2d and viewspace_points to share the same N.")
    dev = m2.device
    gx, gy = tile_grid(int(image_width), int(image_height))
    if int(num_tiles) != gx * gy:
        raise ValueError(f"num_tiles must be {gx * gy} for a {image_width}x{image_height} image")
    t = _raster_tensors(ranges, point_list, per_tile_bucket_offset, means2d, colors, conic_opacity,
                        background, metric_map, metric_count, dev)
    rp = RasterParams(int(image_width), int(image_height), int(num_tiles), int(bucket_sum),
                      int(t["metric_count"].numel()), int(bool(get_flag)))
    outs = _RasterizeFn.apply(rp, t, means2d, colors, conic_opacity, viewspace_points)
    return dict(zip(_RAS_OUT, outs))


def rasterize_backward(ranges, point_list, per_tile_bucket_offset, means2d, colors, conic_opacity,
                       background, dL_dout_color, forward_outputs: dict, image_width: int,
                       image_height: int, num_tiles: int, bucket_sum: int) -> dict:
    """VJP of rasterize_forward for an out_color cotangent [3, H*W]
    (fastgs_core/fastgs_rasterize_backward.cpp:35-166). Returns d_means2d,
    d_colors, d_conic_opacity, d_viewspace_points (the means2D-gradient
    contract: per-Gaussian (sum dL/dx, sum dL/dy, sum |.|, sum |.|))."""
    dev = torch.as_tensor(means2d).device
    n = torch.as_tensor(means2d).shape[0]
    t = _raster_tensors(ranges, point_list, per_tile_bucket_offset, means2d, colors, conic_opacity,
                        background, torch.zeros(1, dtype=torch.int32, device=dev),
                        torch.zeros(n, dtype=torch.int32, device=dev), dev)
    rp = RasterParams(int(image_width), int(image_height), int(num_tiles), int(bucket_sum), n, 0)
    o = {k: forward_outputs[k] for k in ("bucket_to_tile", "sampled_t", "sampled_ar", "final_t",
                                         "n_contrib", "max_contrib", "pixel_colors")}
    o = {k: (v.contiguous() if torch.is_tensor(v) else torch.as_tensor(v, device=dev)) for k, v in o.items()}
    g = _run_rasterize_backward(rp, t, o, _f32(dL_dout_color, dev), dev)
    return dict(d_means2d=g["dmeans2d"], d_colors=g["dcolors"], d_conic_opacity=g["dconic"],
                d_viewspace_points=g["dviewspace"])


# ------------------------------------------------------------------- loss
class _L1DssimFn(torch.autograd.Function):
    """w_l1 * mean|image - target| + w_ssim * (1 - mean SSIM) with its
    gradient from one fused pass (fgs_l1_dssim_loss)."""

    @staticmethod
    def forward(ctx, image, target, w_l1, w_ssim):
        dev = image.device
        if image.dim() != 3 or image.shape[0] != 3 or target.shape != image.shape:
            raise ValueError("l1_dssim_loss expects image and target of shape (3, H, W)")
        H, W = int(image.shape[1]), int(image.shape[2])
        img = _f32(image, dev)
        tgt = _f32(target, dev)
        out = torch.empty(4, dtype=torch.float32, device=dev)
        dimg = torch.empty_like(img)
        scr = _WS.get(dev, "loss", int(lib().fgs_loss_scratch_bytes(W, H)))
        check(lib().fgs_l1_dssim_loss(W, H, _p(img), _p(tgt), float(w_l1), float(w_ssim), _p(out),
                                      _p(dimg), _p(scr), _stream(dev)), "l1_dssim_loss")
        ctx.save_for_backward(dimg)
        return out[0]

    @staticmethod
    def backward(ctx, g):
        (dimg,) = ctx.saved_tensors
        return dimg * g, None, None, None


def l1_dssim_loss(image: torch.Tensor, target: torch.Tensor, w_l1: float = 1.0,
                  w_ssim: float = 0.2) -> torch.Tensor:
    """The training loss of the FastGS trainers with the D-SSIM term
    (scripts/train_scanner_fastgs.py:949-964): w_l1 * mean |image - target| +
    w_ssim * (1 - mean SSIM), SSIM with an 11x11 Gaussian window (sigma 1.5)
    and zero padding. image, target: (3, H, W) float32 CUDA tensors; the
    result is a differentiable scalar w.r.t. image."""
    return _L1DssimFn.apply(image, target, w_l1, w_ssim)


# ------------------------------------------------------ rasterize_gaussians
_DUP_CAP: dict = {}  # device index -> key capacity of the duplicate buffers
_HOST: dict = {}


def _dup_buffers(dev, cap: int):
    k = _WS.get(dev, "dup_keys", cap * 8)[:cap * 8].view(torch.uint64)
    v = _WS.get(dev, "dup_vals", cap * 4)[:cap * 4].view(torch.uint32)
    return k, v


def _duplicate_into(pre, point_offsets, mult, gx, gy, n, cap, dev) -> None:
    keys, vals = _dup_buffers(dev, cap)
    check(lib().fgs_duplicate_with_keys(
        n, float(mult), gx, gy, _p(pre["xys"]), _p(pre["depths"]), _p(point_offsets),
        _p(pre["conic_opacity"]), _p(pre["tiles_touched"]), cap, _p(keys), _p(vals),
        _stream(dev)), "binning_forward")


def _host_slots(dev):
    """Pinned slots for the bucket total and the sort flag, and their event."""
    h = _HOST.get(dev.index)
    if h is None:
        h = _HOST[dev.index] = (torch.empty(1, dtype=torch.int64, pin_memory=True),
                                torch.empty(1, dtype=torch.int32, pin_memory=True),
                                torch.cuda.Event())
    return h


def rasterize_gaussians(inputs: dict, image_width: int, image_height: int, block_x: int = 16,
                        block_y: int = 16, tan_fovx: float = 1.0, tan_fovy: float = 1.0,
                        degree: int = 0, scale_modifier: float = 1.0, mult: float = 1.0,
                        prefiltered: bool = False, get_flag: bool = False) -> dict:
    """The forward chain of binding.cpp:33-282: preprocess -> inclusive scan
    -> duplicate -> sort -> tile prep -> bucket scan -> rasterize. Keys:
    means3d, background, opacities, metric_map, viewmatrix, projmatrix, campos
    (required); colors_precomp (alias colors) XOR dc+sh; cov3d_precomp XOR
    scales+rotations; viewspace_points optional (zeros). Returns the
    reference's 26-entry dict; out_color is differentiable w.r.t. the
    Gaussian inputs and viewspace_points. If nothing is rendered, out_color
    is empty [0] as in the reference."""
    _check_block(block_x, block_y)
    fn = "rasterize_gaussians_forward"
    names = dict(viewmat="viewmatrix", projmat="projmatrix", cam_pos="campos", quats="rotations",
                 aliases=("colors",))
    for k in ("means3d", "background", "opacities", "metric_map", "viewmatrix", "projmatrix", "campos"):
        if k not in inputs:
            raise RuntimeError(f"{fn} missing required input tensor: {k}")
    raw, use_col, use_cov, dev = _prep_inputs(inputs, names, fn)
    W, H = int(image_width), int(image_height)
    n = int(raw["means3d"].shape[0])
    vs = inputs.get("viewspace_points")
    if vs is None or torch.as_tensor(vs).numel() == 0:
        vs = torch.zeros((n, 4), dtype=torch.float32, device=dev)
    pre, _ = _preprocess_apply(raw, W, H, tan_fovx, tan_fovy, degree, scale_modifier, mult,
                               use_col, use_cov, vs, dev)
    gx, gy = tile_grid(W, H)
    T = gx * gy
    point_offsets, total = _scan(pre["tiles_touched"], dev)
    # duplicate-with-keys runs before the host knows K, into per-device
    # grow-only buffers of the capacity earlier calls needed (its writes stop
    # at the capacity); the sort reads them into fresh outputs
    cap = _DUP_CAP.get(dev.index, 0)
    if n and cap:
        _duplicate_into(pre, point_offsets, mult, gx, gy, n, cap, dev)
    num_rendered = int(total.item()) if n else 0  # host sync #1, as binding.cpp:154
    res = {"rendered": num_rendered, "num_buckets": 0}
    empty_f = torch.zeros(0, dtype=torch.float32, device=dev)
    empty_u = torch.zeros(0, dtype=torch.uint32, device=dev)
    metric_count = torch.zeros(n if get_flag else 0, dtype=torch.int32, device=dev)
    point_list_keys = torch.zeros(0, dtype=torch.uint64, device=dev)
    point_list = empty_u
    ranges = torch.zeros((0, 2), dtype=torch.uint32, device=dev)
    bucket_count = empty_u
    bucket_offsets = empty_u
    ras = dict(bucket_to_tile=empty_u, sampled_t=empty_f, sampled_ar=empty_f, final_t=empty_f,
               n_contrib=empty_u, max_contrib=empty_u, pixel_colors=empty_f, out_color=empty_f,
               metric_count=metric_count)
    bucket_sum = 0
    if num_rendered > 0:
        K = num_rendered
        if K > cap:
            cap = _DUP_CAP[dev.index] = K + K // 4 + 1024
            _duplicate_into(pre, point_offsets, mult, gx, gy, n, cap, dev)
        keys_u, vals_u = _dup_buffers(dev, cap)
        st = _stream(dev)
        kb = sort_key_bits(T)
        point_list_keys = torch.empty(K, dtype=torch.uint64, device=dev)
        point_list = torch.empty(K, dtype=torch.uint32, device=dev)
        nbytes = int(lib().fgs_sort_workspace_bytes(K, kb))
        sws = _WS.get(dev, "sort", nbytes)
        check(lib().fgs_sort_pairs(K, kb, _p(keys_u), _p(vals_u), _p(point_list_keys), _p(point_list),
                                   _p(sws), sws.numel(), st), "sort_keys")
        # tile prep with the bucket arrays sized by a bound (every tile has at
        # most n_t/32 + 1 buckets); the bucket total and the sort's timeout
        # flag go to the host on an event while the forward pass renders
        Bmax = (K + 31) // 32 + T
        ranges = torch.empty((T, 2), dtype=torch.uint32, device=dev)
        bucket_count = torch.empty(T, dtype=torch.uint32, device=dev)
        bucket_offsets = torch.empty(T, dtype=torch.uint32, device=dev)
        bsum = torch.empty(1, dtype=torch.uint64, device=dev)
        order = torch.empty(T, dtype=torch.uint32, device=dev)
        b2t = torch.empty(Bmax * 256, dtype=torch.uint32, device=dev)
        check(lib().fgs_tile_prep_ordered(K, T, _p(point_list_keys), _p(ranges), _p(bucket_count),
                                          _p(bucket_offsets), _p(bsum), _p(order), _p(b2t), Bmax, st),
              "tile_prep")
        hb, hf, ev = _host_slots(dev)
        hb.copy_(bsum.view(torch.int64), non_blocking=True)
        hf.copy_(sws[:4].view(torch.int32), non_blocking=True)
        ev.record(torch.cuda.current_stream(dev))
        t = _raster_tensors(ranges, point_list, bucket_offsets, pre["xys"], pre["rgb"],
                            pre["conic_opacity"], inputs["background"], inputs["metric_map"],
                            metric_count, dev)
        t["_tile_order"], t["_bucket_to_tile"] = order, b2t
        rp = RasterParams(W, H, T, Bmax, int(t["metric_count"].numel()), int(bool(get_flag)))
        outs = _RasterizeFn.apply(rp, t, pre["xys"], pre["rgb"], pre["conic_opacity"],
                                  pre["viewspace_points"])
        ev.synchronize()  # host read #2, as binding.cpp:212: the forward pass keeps running
        bucket_sum = int(hb[0])
        if int(hf[0]):
            raise RuntimeError(f"sort_keys failed (status {_lib.FGS_ERR_TIMEOUT}): a look-back "
                               "wait gave up after its poll limit")
        # the backward pass walks the real buckets only
        rp.bucket_sum = bucket_sum
        ras = dict(zip(_RAS_OUT, outs))
        B256 = bucket_sum * 256
        ras["bucket_to_tile"] = b2t[:B256]
        # declared [B*256], only the first B written (fastgs_rasterize.metal:67-75)
        b2t[bucket_sum:B256].zero_()
        ras["sampled_t"] = ras["sampled_t"][:B256]
        ras["sampled_ar"] = ras["sampled_ar"].view(-1)[:3 * B256].view(3, B256)
    res["num_buckets"] = bucket_sum
    res.update({
        "out_color": ras["out_color"], "radii": pre["radii"], "point_offsets": point_offsets,
        "ranges": ranges, "bucket_count": bucket_count, "bucket_offsets": bucket_offsets,
        "point_list_keys": point_list_keys, "point_list": point_list,
        "metric_count": ras["metric_count"], "viewspace_points": pre["viewspace_points"],
        "geom_means2d": pre["xys"], "geom_depths": pre["depths"], "geom_cov3d": pre["cov3d"],
        "geom_rgb": pre["rgb"], "geom_conic_opacity": pre["conic_opacity"],
        "geom_tiles_touched": pre["tiles_touched"], "geom_clamped": pre["clamped"],
        "sample_bucket_to_tile": ras["bucket_to_tile"], "sample_t": ras["sampled_t"],
        "sample_ar": ras["sampled_ar"], "img_final_t": ras["final_t"],
        "img_n_contrib": ras["n_contrib"], "img_max_contrib": ras["max_contrib"],
        "img_pixel_colors": ras["pixel_colors"],
    })
    return res


rasterize_gaussians_forward = rasterize_gaussians
