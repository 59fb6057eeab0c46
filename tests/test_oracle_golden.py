"""The CPU oracle against the golden fixtures made by the reference's own
kernels (tests/golden/make_golden.py) and, where the reference tree was
available to build oracle/_ref, against those kernels directly."""
import hashlib
import os

import numpy as np
import pytest

from fastgs_core_b200 import synthetic as S
from oracle.oracle import Oracle, RefKernels, ref_available

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FWD_FLOAT = ("xys", "depths", "cov3d", "rgb", "conic_opacity", "viewspace_points", "sampled_t",
             "sampled_ar", "final_t", "pixel_colors", "out_color")
FWD_INT = ("radii", "tiles_touched", "clamped", "point_offsets", "point_list_keys_unsorted",
           "point_list_unsorted", "point_list_keys", "point_list", "ranges", "bucket_count",
           "bucket_offsets", "bucket_to_tile", "n_contrib")


def sha(a):
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def _ins(z):
    return {k[3:]: v for k, v in z.items() if k.startswith("in_")}


def rel_err(a, b):
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-12)) if b.size else 0.0


@pytest.mark.parametrize("mode", ["libm", "gpu"])
@pytest.mark.parametrize("case,W,H", [("preprocess_line8", 16, 16), ("e2e16", 32, 32)])
def test_fixture_chain(mode, case, W, H):
    z = load(case)
    o = Oracle(mode)
    f = o.forward(_ins(z), W=W, H=H, tan_fovx=1.0, tan_fovy=1.0, degree=0)
    b = o.backward(f, z["cotangent"])
    for k in FWD_INT:
        if "f_" + k in z:
            assert np.array_equal(f[k], z["f_" + k]), k
    for k in FWD_FLOAT:
        if "f_" + k in z:
            if mode == "libm":
                assert np.array_equal(f[k], z["f_" + k]), k
            else:
                np.testing.assert_allclose(f[k], z["f_" + k], rtol=0, atol=1e-5, err_msg=k)
    for k, v in b.items():
        if mode == "libm":
            assert np.array_equal(v, z["b_" + k]), k
        else:
            assert rel_err(v, z["b_" + k]) < 1e-4, k


@pytest.mark.parametrize("mode", ["libm", "gpu"])
def test_rand_sh3(mode):
    z = load("rand_sh3")
    scene, cam = S.small_scene(11, 300, 3, 40, 24)
    o = Oracle(mode)
    f = o.forward(S.render_inputs(scene, cam, (0.2, 0.1, 0.05)), W=cam.width, H=cam.height,
                  tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, degree=3)
    b = o.backward(f, z["cotangent"])
    for k in FWD_INT:
        assert np.array_equal(f[k], z["f_" + k]), k
    for k in FWD_FLOAT:
        if mode == "libm":
            assert np.array_equal(f[k], z["f_" + k]), k
        else:
            np.testing.assert_allclose(f[k], z["f_" + k], rtol=0, atol=1e-5, err_msg=k)
    for k, v in b.items():
        if mode == "libm":
            assert np.array_equal(v, z["b_" + k]), k
        else:
            assert rel_err(v, z["b_" + k]) < 1e-3, k


def test_tile_prep_hand():
    z = load("tile_prep_hand")
    np.testing.assert_array_equal(z["ranges"], [[0, 2], [2, 5], [0, 0], [5, 8]])
    np.testing.assert_array_equal(z["bucket_count"], [1, 1, 0, 1])
    r = np.zeros((4, 2), np.uint32)
    bc = np.zeros(4, np.uint32)
    Oracle("gpu").tile_prep(8, 4, z["keys"], r, bc)
    assert np.array_equal(r, z["ranges"]) and np.array_equal(bc, z["bucket_count"])


def test_raster_one_splat():
    z = load("raster_one")
    o = Oracle("libm")
    a = dict(ranges=np.array([[0, 1]], np.uint32), point_list=np.array([0], np.uint32),
             bucket_offsets=np.array([1], np.uint32), means2d=z["means2d"], colors=z["colors"],
             conic_opacity=z["conic_opacity"], background=np.zeros(3, np.float32),
             metric_map=np.zeros(256, np.int32), bucket_to_tile=np.zeros(256, np.uint32),
             sampled_t=np.zeros(256, np.float32), sampled_ar=np.zeros(3 * 256, np.float32),
             final_t=np.zeros(256, np.float32), n_contrib=np.zeros(256, np.uint32),
             max_contrib=np.zeros(1, np.uint32), pixel_colors=np.zeros((3, 256), np.float32),
             out_color=np.zeros((3, 256), np.float32), metric_count=np.zeros(0, np.int32),
             metric_count_buf=np.zeros(1, np.int32))
    o.render_forward(16, 16, 1, 1, 0, a)
    for k in ("bucket_to_tile", "sampled_t", "sampled_ar", "final_t", "n_contrib", "max_contrib",
              "pixel_colors", "out_color"):
        assert np.array_equal(a[k], z[k]), k
    g = dict(dL_dout=z["dL_dout"], dmeans2d=np.zeros((1, 2), np.float32),
             dcolors=np.zeros((1, 3), np.float32), dconic=np.zeros((1, 4), np.float32),
             dviewspace=np.zeros((1, 4), np.float32))
    o.render_backward(16, 16, 1, 1, a, g)
    for k in ("dmeans2d", "dcolors", "dconic", "dviewspace"):
        assert np.array_equal(g[k], z[k]), k


def test_config1_hashes():
    lines = open(os.path.join(GOLD, "config1.sha256")).read().split("\n")
    want = {}
    for ln in lines:
        p = ln.split()
        if len(p) == 3:
            want[(p[0], p[1])] = p[2]
        elif len(p) == 2:
            want[p[0]] = int(p[1])
    scene, cams = S.config1(0)
    cam = cams[0]
    o = Oracle("libm", threads=4)
    f = o.forward(S.render_inputs(scene, cam), W=cam.width, H=cam.height, tan_fovx=cam.tan_fovx,
                  tan_fovy=cam.tan_fovy, degree=0)
    assert f["rendered"] == want["rendered"] and f["num_buckets"] == want["num_buckets"]
    hashes = [(k, v) for k, v in want.items() if isinstance(k, tuple)]
    for (kind, k), h in hashes:
        if kind == "fwd":
            assert sha(f[k]) == h, k
    o.set_threads(1)  # deterministic float atomics order for the hash comparison
    w = np.random.default_rng(4).uniform(-1, 1, (3, cam.width * cam.height)).astype(np.float32)
    b = o.backward(f, w)
    for (kind, k), h in hashes:
        if kind == "bwd":
            assert sha(b[k]) == h, k


def test_config1_samples_gpu_mode():
    """The GPU-mode oracle (shared exp/log) against the reference on config 1."""
    z = load("config1_samples")
    scene, cams = S.config1(0)
    cam = cams[0]
    o = Oracle("gpu", threads=4)
    f = o.forward(S.render_inputs(scene, cam), W=cam.width, H=cam.height, tan_fovx=cam.tan_fovx,
                  tan_fovy=cam.tan_fovy, degree=0)
    assert np.array_equal(f["tiles_touched"][z["gi"]], z["tiles_touched"])
    assert np.array_equal(f["radii"][z["gi"]], z["radii"])
    np.testing.assert_allclose(f["out_color"][:, z["pix"]], z["out_color"], atol=1e-4, rtol=0)
    o.set_threads(1)
    w = np.random.default_rng(4).uniform(-1, 1, (3, cam.width * cam.height)).astype(np.float32)
    b = o.backward(f, w)
    for k in ("dmeans3d", "dscales", "dquats", "dopacities", "ddc"):
        assert rel_err(b[k][z["gi"]], z[k]) < 1e-3, k


@pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built (no reference tree)")
@pytest.mark.parametrize("seed,n,deg,W,H", [(21, 200, 1, 33, 17), (22, 500, 2, 48, 48),
                                            (23, 400, 3, 64, 40)])
def test_oracle_libm_equals_reference(seed, n, deg, W, H):
    scene, cam = S.small_scene(seed, n, deg, W, H, log_scale_mu=-2.8)
    ins = S.render_inputs(scene, cam, (0.3, 0.3, 0.3))
    kw = dict(W=W, H=H, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, degree=deg)
    r = RefKernels().forward(ins, **kw)
    o = Oracle("libm").forward(ins, **kw)
    full_tiles = (W % 16 == 0) and (H % 16 == 0)
    for k in FWD_INT + FWD_FLOAT + (("max_contrib",) if full_tiles else ()):
        assert np.array_equal(r[k], o[k]), k
    w = np.random.default_rng(seed).standard_normal((3, W * H)).astype(np.float32)
    rb = RefKernels().backward(r, w)
    ob = Oracle("libm").backward(o, w)
    for k in rb:
        assert np.array_equal(rb[k], ob[k]), k


def test_exp_log_accuracy():
    o = Oracle("gpu")
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-87, 0, 2000), rng.uniform(-6, 0, 2000), [0.0, -1e-8, -86.9]])
    for x in xs.astype(np.float32):
        want = np.exp(np.float64(x))
        got = o.expf(float(x))
        assert abs(got - want) <= 2.5 * np.spacing(np.float32(want)), (x, got, want)
    ys = np.concatenate([rng.uniform(1e-3, 300, 2000), 10 ** rng.uniform(-30, 30, 2000), [1.0, 255.0]])
    for y in ys.astype(np.float32):
        want = np.log(np.float64(y))
        got = o.logf(float(y))
        assert abs(got - want) <= 2.5 * np.spacing(np.float32(abs(want)) if want != 0 else np.float32(1e-30)), (y, got, want)
    assert o.expf(-100.0) == 0.0 and o.logf(0.0) == -np.inf and np.isnan(o.logf(-1.0))


def test_oracle_sort_matches_stable_argsort():
    rng = np.random.default_rng(3)
    k = 50000
    tiles = rng.integers(0, 5000, k).astype(np.uint64)
    depth = rng.uniform(0.2, 50, k).astype(np.float32).view(np.uint32).astype(np.uint64)
    depth[::7] = depth[0]  # ties
    keys = (tiles << np.uint64(32)) | depth
    vals = np.arange(k, dtype=np.uint32)
    sk, sv = Oracle("gpu").sort(keys, vals, 45)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(sk, keys[order]) and np.array_equal(sv, vals[order])
