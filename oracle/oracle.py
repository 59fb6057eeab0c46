"""Python driver for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm import this module, as the checker or the timed CPU baseline.

Two back ends share one orchestration that follows the reference's forward
chain (fastgs_core/binding/binding.cpp:33-282: preprocess -> inclusive cumsum
-> duplicate -> stable argsort/take -> tile prep -> cumsum of bucket counts ->
render) and its VJP chain (fastgs_core/fastgs_rasterize.cpp:191-206 ->
fastgs_rasterize_backward.cpp:35-75, then fastgs_preprocess.cpp:191-206 ->
fastgs_preprocess_backward.cpp:39-79):

* ``Oracle(mode="gpu")``  - fgs_oracle.c with the exp/log definition the CUDA
  kernels share (bit-identical integer outputs and image vs the GPU);
* ``Oracle(mode="libm")`` - the same C with libm exp/log;
* ``RefKernels()``        - the reference's own Metal kernels compiled for this
  CPU (oracle/_ref, built by oracle/build.py where the reference tree exists).

All arrays are numpy, float32 / uint32 / int32 / uint64 / bool, in the
reference's layouts.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_f = C.c_float
_i = C.c_int
_i64 = C.c_int64
_p = C.c_void_p


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def _c(a, dt) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dt))


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libfgs_ref.so"))


class _Backend:
    """Common orchestration; subclasses bind the per-stage kernels."""

    name = "base"

    # ------------------------------------------------------------- stages
    def preprocess(self, n, degree, maxc, scale_mod, mult, tanx, tany, W, H, use_cov, use_col, ins):
        raise NotImplementedError

    def duplicate(self, n, mult, gx, gy, xys, depths, offsets, conic, tiles, keys, vals):
        raise NotImplementedError

    def sort(self, keys, vals, key_bits):
        raise NotImplementedError

    def tile_prep(self, K, T, keys, ranges, bucket_count):
        raise NotImplementedError

    def render_forward(self, W, H, T, B, get_flag, a):
        raise NotImplementedError

    def render_backward(self, W, H, T, B, a, g):
        raise NotImplementedError

    def preprocess_backward(self, n, W, H, use_cov, use_col, scale_mod, tanx, tany, degree, maxc, a, g):
        raise NotImplementedError

    # -------------------------------------------------------- orchestration
    def forward(self, inputs: dict, W: int, H: int, tan_fovx: float, tan_fovy: float,
                degree: int = 0, scale_modifier: float = 1.0, mult: float = 1.0,
                get_flag: bool = False) -> dict:
        """Forward chain of binding.cpp:33-282. ``inputs`` uses the
        rasterize_gaussians key names (means3d, opacities, dc+sh or
        colors_precomp, scales+rotations or cov3d_precomp, viewmatrix,
        projmatrix, campos, background, metric_map, viewspace_points)."""
        means3d = _c(inputs["means3d"], np.float32)
        n = means3d.shape[0]
        use_col = "colors_precomp" in inputs
        use_cov = "cov3d_precomp" in inputs
        dc = _c(inputs["dc"], np.float32) if not use_col else np.zeros((n, 3), np.float32)
        sh = _c(inputs["sh"], np.float32) if not use_col else np.zeros((n, 0, 3), np.float32)
        maxc = sh.shape[1] if sh.ndim >= 2 else 0
        vs = inputs.get("viewspace_points")
        vs = np.zeros((n, 4), np.float32) if vs is None else _c(vs, np.float32)
        ins = dict(
            means3d=means3d, dc=dc, sh=sh,
            colors_precomp=_c(inputs["colors_precomp"], np.float32) if use_col else np.zeros((n, 3), np.float32),
            opacities=_c(inputs["opacities"], np.float32).reshape(n),
            scales=_c(inputs["scales"], np.float32) if not use_cov else np.zeros((n, 3), np.float32),
            rotations=_c(inputs["rotations"], np.float32) if not use_cov else np.zeros((n, 4), np.float32),
            cov3d_precomp=_c(inputs["cov3d_precomp"], np.float32) if use_cov else np.zeros((n, 6), np.float32),
            viewmatrix=_c(inputs["viewmatrix"], np.float32),
            projmatrix=_c(inputs["projmatrix"], np.float32),
            campos=_c(inputs["campos"], np.float32).reshape(-1),
            viewspace_points=vs,
        )
        pre = self.preprocess(n, degree, maxc, scale_modifier, mult, tan_fovx, tan_fovy, W, H,
                              int(use_cov), int(use_col), ins)
        gx, gy = (W + 15) // 16, (H + 15) // 16
        T = gx * gy
        offsets = np.cumsum(pre["tiles_touched"], dtype=np.uint32)
        K = int(offsets[-1]) if n else 0
        out = dict(pre)
        out["point_offsets"] = offsets
        out["rendered"] = K
        background = _c(inputs["background"], np.float32).reshape(3)
        metric_map = _c(inputs.get("metric_map", np.zeros(W * H, np.int32)), np.int32).reshape(-1)
        if K == 0:
            out.update(point_list_keys=np.zeros(0, np.uint64), point_list=np.zeros(0, np.uint32),
                       ranges=np.zeros((0, 2), np.uint32), bucket_count=np.zeros(0, np.uint32),
                       bucket_offsets=np.zeros(0, np.uint32), num_buckets=0,
                       out_color=np.zeros(0, np.float32))
            return out
        keys = np.zeros(K, np.uint64)
        vals = np.zeros(K, np.uint32)
        self.duplicate(n, mult, gx, gy, pre["xys"], pre["depths"], offsets, pre["conic_opacity"],
                       pre["tiles_touched"], keys, vals)
        out["point_list_keys_unsorted"] = keys.copy()
        out["point_list_unsorted"] = vals.copy()
        key_bits = 32 + max(1, int(T - 1).bit_length())
        keys, vals = self.sort(keys, vals, key_bits)
        ranges = np.zeros((T, 2), np.uint32)
        bucket_count = np.zeros(T, np.uint32)
        self.tile_prep(K, T, keys, ranges, bucket_count)
        bucket_offsets = np.cumsum(bucket_count, dtype=np.uint32)
        B = int(bucket_offsets[-1])
        out.update(point_list_keys=keys, point_list=vals, ranges=ranges, bucket_count=bucket_count,
                   bucket_offsets=bucket_offsets, num_buckets=B)
        if B == 0:
            out["out_color"] = np.zeros(0, np.float32)
            return out
        P = W * H
        a = dict(ranges=ranges, point_list=vals, bucket_offsets=bucket_offsets,
                 means2d=pre["xys"], colors=pre["rgb"], conic_opacity=pre["conic_opacity"],
                 background=background, radii=pre["radii"], metric_map=metric_map,
                 bucket_to_tile=np.zeros(B * 256, np.uint32),
                 sampled_t=np.zeros(B * 256, np.float32),
                 # +96 floats: the reference backward reads one 32-wide chunk
                 # past the end of the last bucket (fastgs_rasterize_backward.metal:115-126)
                 sampled_ar=np.zeros(3 * B * 256 + 96, np.float32),
                 final_t=np.zeros(P, np.float32), n_contrib=np.zeros(P, np.uint32),
                 max_contrib=np.zeros(T, np.uint32), pixel_colors=np.zeros((3, P), np.float32),
                 out_color=np.zeros((3, P), np.float32),
                 metric_count=np.zeros(n if get_flag else 0, np.int32))
        if not get_flag:
            a["metric_count_buf"] = np.zeros(max(n, 1), np.int32)
        self.render_forward(W, H, T, B, int(get_flag), a)
        out.update(bucket_to_tile=a["bucket_to_tile"], sampled_t=a["sampled_t"],
                   sampled_ar=a["sampled_ar"][: 3 * B * 256].reshape(3, B * 256),
                   final_t=a["final_t"], n_contrib=a["n_contrib"], max_contrib=a["max_contrib"],
                   pixel_colors=a["pixel_colors"], out_color=a["out_color"],
                   metric_count=a["metric_count"], _raster=a, _ins=ins, _W=W, _H=H,
                   _params=dict(degree=degree, maxc=maxc, scale_modifier=scale_modifier,
                                tan_fovx=tan_fovx, tan_fovy=tan_fovy, use_cov=int(use_cov),
                                use_col=int(use_col)))
        return out

    def backward(self, fwd: dict, dL_dout_color: np.ndarray) -> dict:
        """VJP of the forward chain for a cotangent on out_color [3, H*W].
        Returns the rasterize-level grads (means2d, colors, conic_opacity,
        viewspace) and the preprocess-level grads w.r.t. the primal inputs."""
        a = fwd["_raster"]
        ins = fwd["_ins"]
        p = fwd["_params"]
        W, H = fwd["_W"], fwd["_H"]
        n = ins["means3d"].shape[0]
        T = a["ranges"].shape[0]
        B = fwd["num_buckets"]
        g = dict(dL_dout=_c(dL_dout_color, np.float32).reshape(3, W * H),
                 dmeans2d=np.zeros((n, 2), np.float32), dcolors=np.zeros((n, 3), np.float32),
                 dconic=np.zeros((n, 4), np.float32), dviewspace=np.zeros((n, 4), np.float32))
        self.render_backward(W, H, T, B, a, g)
        pg = dict(dcov3d=np.zeros((n, 6), np.float32), drgb=g["dcolors"], dxys=g["dmeans2d"],
                  dconic=g["dconic"], dvs=g["dviewspace"], ddepths=np.zeros(n, np.float32),
                  dmeans3d=np.zeros((n, 3), np.float32), ddc=np.zeros((n, 3), np.float32),
                  dsh=np.zeros_like(ins["sh"]), dcolors_precomp=np.zeros((n, 3), np.float32),
                  dopacities=np.zeros(n, np.float32), dscales=np.zeros((n, 3), np.float32),
                  dquats=np.zeros((n, 4), np.float32), dvs_in=np.zeros((n, 4), np.float32))
        pa = dict(ins=ins, cov3d=fwd["cov3d"], radii=fwd["radii"], clamped=fwd["clamped"])
        self.preprocess_backward(n, W, H, p["use_cov"], p["use_col"], p["scale_modifier"],
                                 p["tan_fovx"], p["tan_fovy"], p["degree"], p["maxc"], pa, pg)
        return dict(dmeans2d=g["dmeans2d"], dcolors=g["dcolors"], dconic_opacity=g["dconic"],
                    dviewspace_raster=g["dviewspace"], dmeans3d=pg["dmeans3d"], ddc=pg["ddc"],
                    dsh=pg["dsh"], dcolors_precomp=pg["dcolors_precomp"],
                    dopacities=pg["dopacities"], dscales=pg["dscales"], dquats=pg["dquats"],
                    dviewspace_points=pg["dvs_in"])


def _new_pre_outputs(n):
    return dict(radii=np.zeros(n, np.int32), xys=np.zeros((n, 2), np.float32),
                depths=np.zeros(n, np.float32), cov3d=np.zeros((n, 6), np.float32),
                rgb=np.zeros((n, 3), np.float32), conic_opacity=np.zeros((n, 4), np.float32),
                tiles_touched=np.zeros(n, np.uint32), clamped=np.zeros((n, 3), np.bool_),
                viewspace_points=np.zeros((n, 4), np.float32))


class Oracle(_Backend):
    """fgs_oracle.c through ctypes. ``mode`` is "gpu" (the exp/log the CUDA
    kernels share) or "libm"."""

    def __init__(self, mode: str = "gpu", threads: int = 1):
        lib = "liboracle.so" if mode == "gpu" else "liboracle_libm.so"
        path = os.path.join(HERE, lib)
        if not os.path.exists(path):
            from oracle import build as _b  # noqa: WPS433

            _b.build_oracle()
        self.lib = C.CDLL(path)
        self.name = f"oracle-{mode}"
        self.lib.o_fgs_expf.restype = _f
        self.lib.o_fgs_expf.argtypes = [_f]
        self.lib.o_fgs_logf.restype = _f
        self.lib.o_fgs_logf.argtypes = [_f]
        self.set_threads(threads)

    def set_threads(self, n: int) -> None:
        self.lib.o_set_threads(_i(int(n)))

    def expf(self, x: float) -> float:
        return self.lib.o_fgs_expf(_f(x))

    def logf(self, x: float) -> float:
        return self.lib.o_fgs_logf(_f(x))

    def preprocess(self, n, degree, maxc, scale_mod, mult, tanx, tany, W, H, use_cov, use_col, ins):
        o = _new_pre_outputs(n)
        self.lib.o_preprocess_forward(
            _i(n), _i(degree), _i(maxc), _f(scale_mod), _f(mult), _f(tanx), _f(tany), _i(W), _i(H),
            _i(use_cov), _i(use_col), *[_p(_ptr(ins[k])) for k in (
                "means3d", "dc", "sh", "colors_precomp", "opacities", "scales", "rotations",
                "cov3d_precomp", "viewmatrix", "projmatrix", "campos", "viewspace_points")],
            *[_p(_ptr(o[k])) for k in ("radii", "xys", "depths", "cov3d", "rgb", "conic_opacity",
                                       "tiles_touched", "clamped", "viewspace_points")])
        return o

    def duplicate(self, n, mult, gx, gy, xys, depths, offsets, conic, tiles, keys, vals):
        self.lib.o_duplicate_with_keys(_i(n), _f(mult), _i(gx), _i(gy), _p(_ptr(xys)), _p(_ptr(depths)),
                                       _p(_ptr(offsets)), _p(_ptr(conic)), _p(_ptr(tiles)),
                                       _p(_ptr(keys)), _p(_ptr(vals)))

    def sort(self, keys, vals, key_bits):
        keys = keys.copy()
        vals = vals.copy()
        tk = np.empty_like(keys)
        tv = np.empty_like(vals)
        self.lib.o_sort_pairs(_i64(keys.size), _i(key_bits), _p(_ptr(keys)), _p(_ptr(vals)),
                              _p(_ptr(tk)), _p(_ptr(tv)))
        return keys, vals

    def tile_prep(self, K, T, keys, ranges, bucket_count):
        self.lib.o_tile_prep(_i64(K), _i(T), _p(_ptr(keys)), _p(_ptr(ranges)), _p(_ptr(bucket_count)))

    def render_forward(self, W, H, T, B, get_flag, a):
        mc = a["metric_count"] if get_flag else a["metric_count_buf"]
        self.lib.o_render_forward(
            _i(W), _i(H), _i(get_flag), *[_p(_ptr(a[k])) for k in (
                "ranges", "point_list", "bucket_offsets", "means2d", "colors", "conic_opacity",
                "background", "metric_map", "bucket_to_tile", "sampled_t", "sampled_ar",
                "final_t", "n_contrib", "max_contrib", "pixel_colors", "out_color")], _p(_ptr(mc)))

    def render_backward(self, W, H, T, B, a, g):
        self.lib.o_render_backward(
            _i(W), _i(H), _i(B), *[_p(_ptr(a[k])) for k in (
                "ranges", "point_list", "bucket_offsets", "means2d", "colors", "conic_opacity",
                "background")], _p(_ptr(g["dL_dout"])), *[_p(_ptr(a[k])) for k in (
                "bucket_to_tile", "sampled_t", "sampled_ar", "final_t", "n_contrib",
                "max_contrib", "pixel_colors")],
            *[_p(_ptr(g[k])) for k in ("dmeans2d", "dcolors", "dconic", "dviewspace")])

    def preprocess_backward(self, n, W, H, use_cov, use_col, scale_mod, tanx, tany, degree, maxc, a, g):
        ins = a["ins"]
        self.lib.o_preprocess_backward(
            _i(n), _i(W), _i(H), _i(use_cov), _i(use_col), _f(scale_mod), _f(tanx), _f(tany),
            _i(degree), _i(maxc), *[_p(_ptr(ins[k])) for k in (
                "means3d", "scales", "rotations", "viewmatrix", "projmatrix", "campos", "sh",
                "cov3d_precomp")], _p(_ptr(a["cov3d"])),
            *[_p(_ptr(g[k])) for k in ("dcov3d", "drgb", "dxys", "dconic", "dvs")],
            _p(_ptr(a["radii"])), _p(_ptr(a["clamped"])),
            *[_p(_ptr(g[k])) for k in ("dmeans3d", "ddc", "dsh", "dcolors_precomp", "dopacities",
                                       "dscales", "dquats", "dvs_in")])


class RefKernels(_Backend):
    """The reference's own Metal kernels compiled for this CPU (oracle/_ref)."""

    name = "reference"

    def __init__(self):
        path = os.path.join(HERE, "_ref", "libfgs_ref.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path + " (run python oracle/build.py where the reference tree exists)")
        self.lib = C.CDLL(path)

    def preprocess(self, n, degree, maxc, scale_mod, mult, tanx, tany, W, H, use_cov, use_col, ins):
        o = _new_pre_outputs(n)
        self.lib.ref_preprocess_forward(
            _i(n), _i(degree), _i(maxc), _f(scale_mod), _f(mult), _f(tanx), _f(tany), _i(W), _i(H),
            _i(0), _i(use_cov), _i(use_col), *[_p(_ptr(ins[k])) for k in (
                "means3d", "dc", "sh", "colors_precomp", "opacities", "scales", "rotations",
                "cov3d_precomp", "viewmatrix", "projmatrix", "campos", "viewspace_points")],
            *[_p(_ptr(o[k])) for k in ("radii", "xys", "depths", "cov3d", "rgb", "conic_opacity",
                                       "tiles_touched", "clamped", "viewspace_points")])
        return o

    def duplicate(self, n, mult, gx, gy, xys, depths, offsets, conic, tiles, keys, vals):
        self.lib.ref_duplicate_with_keys(_i(n), _f(mult), _i(gx), _i(gy), _p(_ptr(xys)), _p(_ptr(depths)),
                                         _p(_ptr(offsets)), _p(_ptr(conic)), _p(_ptr(tiles)),
                                         _p(_ptr(keys)), _p(_ptr(vals)))

    def sort(self, keys, vals, key_bits):
        # binding.cpp:195-197 sorts with mx::argsort; the stable order is the
        # one defined for ties (keys are unique unless two depths are equal)
        order = np.argsort(keys, kind="stable")
        return np.ascontiguousarray(keys[order]), np.ascontiguousarray(vals[order])

    def tile_prep(self, K, T, keys, ranges, bucket_count):
        self.lib.ref_tile_prep(_i(K), _i(T), _p(_ptr(keys)), _p(_ptr(ranges)), _p(_ptr(bucket_count)))

    def render_forward(self, W, H, T, B, get_flag, a):
        mc = a["metric_count"] if get_flag else a["metric_count_buf"]
        self.lib.ref_render_forward(
            _i(W), _i(H), _i(T), _i(B), _i(get_flag), *[_p(_ptr(a[k])) for k in (
                "ranges", "point_list", "bucket_offsets", "means2d", "colors", "conic_opacity",
                "background", "radii", "metric_map", "bucket_to_tile", "sampled_t", "sampled_ar",
                "final_t", "n_contrib", "max_contrib", "pixel_colors", "out_color")], _p(_ptr(mc)))

    def render_backward(self, W, H, T, B, a, g):
        self.lib.ref_render_backward(
            _i(W), _i(H), _i(T), _i(B), *[_p(_ptr(a[k])) for k in (
                "ranges", "point_list", "bucket_offsets", "means2d", "colors", "conic_opacity",
                "background")], _p(_ptr(g["dL_dout"])), *[_p(_ptr(a[k])) for k in (
                "bucket_to_tile", "sampled_t", "sampled_ar", "final_t", "n_contrib",
                "max_contrib", "pixel_colors")],
            *[_p(_ptr(g[k])) for k in ("dmeans2d", "dcolors", "dconic", "dviewspace")])

    def preprocess_backward(self, n, W, H, use_cov, use_col, scale_mod, tanx, tany, degree, maxc, a, g):
        ins = a["ins"]
        self.lib.ref_preprocess_backward(
            _i(n), _i(W), _i(H), _i(use_cov), _i(use_col), _f(scale_mod), _f(tanx), _f(tany),
            _i(degree), _i(maxc), *[_p(_ptr(ins[k])) for k in (
                "means3d", "scales", "rotations", "viewmatrix", "projmatrix", "campos", "sh",
                "cov3d_precomp")], _p(_ptr(a["cov3d"])),
            *[_p(_ptr(g[k])) for k in ("dcov3d", "drgb", "dxys", "ddepths", "dconic", "dvs")],
            _p(_ptr(a["radii"])), _p(_ptr(a["clamped"])),
            *[_p(_ptr(g[k])) for k in ("dmeans3d", "ddc", "dsh", "dcolors_precomp", "dopacities",
                                       "dscales", "dquats", "dvs_in")])
