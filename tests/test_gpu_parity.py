"""GPU parity: the CUDA path (through the public API / C ABI) against the CPU
oracle (mode "gpu": the exp/log definition the kernels share).

Bar: integer outputs (tiles touched, keys, point list, ranges, bucket counts,
n_contrib, max_contrib) and every forward float output (including the
rendered image) bit-identical; gradients within 1e-3 relative (the order of
the float atomics differs)."""
import numpy as np
import pytest
import torch

import fastgs_core_b200 as fg
from fastgs_core_b200 import synthetic as S
from oracle.oracle import Oracle
from tests._gpu_util import GEOM, GRAD_MAP, INT_KEYS, rel_err, run_chain

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3

CASES = [
    # seed, n, degree, W, H, log-scale mean, opacity-logit mean, background
    (1, 300, 0, 32, 32, -3.0, 0.0, (0.0, 0.0, 0.0)),
    (2, 800, 3, 64, 40, -3.0, -1.0, (0.1, 0.2, 0.3)),       # partial tile row
    (3, 1500, 2, 100, 75, -2.5, 1.0, (1.0, 1.0, 1.0)),      # partial tiles both axes
    (4, 3000, 3, 128, 128, -3.5, 2.0, (0.5, 0.0, 0.25)),    # many opaque splats: early stop
    (5, 600, 1, 17, 200, -2.0, 0.0, (0.0, 0.0, 0.0)),       # tall narrow image, big splats
]


def _oracle(ins, W, H, cam, deg, cot, get_flag=False):
    o = Oracle("gpu")
    f = o.forward(ins, W=W, H=H, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, degree=deg,
                  get_flag=get_flag)
    b = o.backward(f, cot) if f.get("num_buckets", 0) else {}
    return f, b


def _compare(res, f, grads=None, b=None):
    assert res["rendered"] == f["rendered"]
    assert res["num_buckets"] == f["num_buckets"]
    for k in INT_KEYS:
        assert np.array_equal(res[k], f[k]), k
    for k, ok in GEOM.items():
        assert np.array_equal(res[k], f[ok]), k
    assert np.array_equal(res["out_color"], f["out_color"]), "out_color"
    B = f["num_buckets"]
    assert np.array_equal(res["sample_bucket_to_tile"][:B], f["bucket_to_tile"][:B])
    assert not res["sample_bucket_to_tile"][B:].any()
    if grads is not None:
        for k, g in grads.items():
            want = b[GRAD_MAP[k]].reshape(g.shape)
            assert rel_err(g, want) < GRAD_TOL, (k, rel_err(g, want))


@pytest.mark.parametrize("case", CASES, ids=[f"c{c[0]}" for c in CASES])
def test_chain_parity(case, cuda_dev):
    seed, n, deg, W, H, ls, om, bg = case
    scene, cam = S.small_scene(seed, n, deg, W, H, log_scale_mu=ls, op_mu=om)
    ins = S.render_inputs(scene, cam, bg)
    cot = np.random.default_rng(seed).standard_normal((3, W * H)).astype(np.float32)
    res, grads = run_chain(ins, W, H, cam.tan_fovx, cam.tan_fovy, deg, cuda_dev, cot)
    f, b = _oracle(ins, W, H, cam, deg, cot)
    _compare(res, f, grads, b)


def test_golden_e2e16_precomp_paths(cuda_dev):
    import os
    z = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "e2e16.npz")))
    ins = {k[3:]: v for k, v in z.items() if k.startswith("in_")}
    res, grads = run_chain(ins, 32, 32, 1.0, 1.0, 0, cuda_dev, z["cotangent"])
    for k in ("radii", "point_list_keys", "point_list", "ranges"):
        assert np.array_equal(res[k], z["f_" + k]), k
    assert np.array_equal(res["img_n_contrib"], z["f_n_contrib"])
    np.testing.assert_allclose(res["out_color"], z["f_out_color"], atol=1e-5, rtol=0)
    assert rel_err(grads["means3d"], z["b_dmeans3d"]) < GRAD_TOL
    assert rel_err(grads["colors_precomp"], z["b_dcolors_precomp"]) < GRAD_TOL
    assert rel_err(grads["opacities"], z["b_dopacities"]) < GRAD_TOL
    assert rel_err(grads["viewspace_points"], z["b_dviewspace_points"]) < GRAD_TOL
    assert not grads["cov3d_precomp"].any()  # the reference never writes d(cov3d_precomp)


def test_golden_rand_sh3(cuda_dev):
    import os
    z = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "rand_sh3.npz")))
    scene, cam = S.small_scene(11, 300, 3, 40, 24)
    ins = S.render_inputs(scene, cam, (0.2, 0.1, 0.05))
    res, grads = run_chain(ins, 40, 24, cam.tan_fovx, cam.tan_fovy, 3, cuda_dev, z["cotangent"])
    for k in ("radii", "point_offsets", "point_list_keys", "point_list", "ranges", "bucket_count"):
        assert np.array_equal(res[k], z["f_" + k]), k
    assert np.array_equal(res["img_n_contrib"], z["f_n_contrib"])
    np.testing.assert_allclose(res["out_color"], z["f_out_color"], atol=1e-4, rtol=0)
    for k in ("means3d", "dc", "sh", "opacities", "scales", "rotations"):
        assert rel_err(grads[k], z["b_" + GRAD_MAP[k]].reshape(grads[k].shape)) < GRAD_TOL, k


def test_metric_count_get_flag(cuda_dev):
    scene, cam = S.small_scene(8, 1000, 0, 64, 64, log_scale_mu=-2.5)
    ins = S.render_inputs(scene, cam)
    rng = np.random.default_rng(8)
    ins["metric_map"] = (rng.uniform(size=64 * 64) < 0.3).astype(np.int32)
    res, _ = run_chain(ins, 64, 64, cam.tan_fovx, cam.tan_fovy, 0, cuda_dev, None, get_flag=True)
    f = Oracle("gpu").forward(ins, W=64, H=64, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy,
                              degree=0, get_flag=True)
    assert res["metric_count"].sum() > 0
    assert np.array_equal(res["metric_count"], f["metric_count"])


def test_nothing_rendered(cuda_dev):
    scene, cam = S.small_scene(9, 50, 0, 32, 32)
    ins = S.render_inputs(scene, cam)
    ins["means3d"] = (cam.campos[None, :] * 3.0 + 0 * ins["means3d"]).astype(np.float32)  # all behind
    res, _ = run_chain(ins, 32, 32, cam.tan_fovx, cam.tan_fovy, 0, cuda_dev, None)
    assert res["rendered"] == 0 and res["num_buckets"] == 0
    assert res["out_color"].size == 0
    assert not res["radii"].any()


def test_empty_input(cuda_dev):
    """N = 0: the reference's path checks see empty scales/rotations as
    missing (binding.cpp:80-89), so the call is rejected the same way."""
    scene, cam = S.small_scene(9, 1, 0, 32, 32)
    ins = S.render_inputs(scene, cam)
    for k in ("means3d", "dc", "sh", "opacities", "scales", "rotations", "viewspace_points"):
        ins[k] = ins[k][:0]
    with pytest.raises(RuntimeError, match="exactly one geometry path"):
        run_chain(ins, 32, 32, cam.tan_fovx, cam.tan_fovy, 0, cuda_dev, None)
    # with the cov3d_precomp path an empty scene renders nothing
    del ins["scales"], ins["rotations"]
    ins["cov3d_precomp"] = np.zeros((0, 6), np.float32)
    with pytest.raises(RuntimeError, match="exactly one geometry path"):
        run_chain(ins, 32, 32, cam.tan_fovx, cam.tan_fovy, 0, cuda_dev, None)


def test_preprocess_forward_api_line8(cuda_dev):
    import os
    z = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "preprocess_line8.npz")))
    ins = {k[3:]: torch.from_numpy(v).to(cuda_dev) for k, v in z.items() if k.startswith("in_")}
    d = dict(means3d=ins["means3d"], opacities=ins["opacities"], cov3d_precomp=ins["cov3d_precomp"],
             colors_precomp=ins["colors_precomp"], viewmat=ins["viewmatrix"],
             projmat=ins["projmatrix"], cam_pos=ins["campos"],
             viewspace_points=ins["viewspace_points"])
    out = fg.preprocess_forward(d, 16, 16)
    for k in ("radii", "tiles_touched", "clamped"):
        assert np.array_equal(out[k].cpu().numpy(), z["f_" + k]), k
    for k in ("xys", "depths", "cov3d", "rgb", "conic_opacity", "viewspace_points"):
        np.testing.assert_allclose(out[k].cpu().numpy(), z["f_" + k], atol=1e-6, rtol=1e-6, err_msg=k)


def test_tile_prep_hand_keys(cuda_dev):
    keys = torch.tensor([(0 << 32) | 1, (0 << 32) | 2, (1 << 32) | 1, (1 << 32) | 2, (1 << 32) | 3,
                         (3 << 32) | 1, (3 << 32) | 2, (3 << 32) | 3], dtype=torch.uint64).to(cuda_dev)
    out = fg.tile_prep_forward(keys, 8, 4)
    assert out["ranges"].cpu().numpy().tolist() == [[0, 2], [2, 5], [0, 0], [5, 8]]
    assert out["bucket_count"].cpu().numpy().tolist() == [1, 1, 0, 1]


@pytest.mark.parametrize("k", [1, 2, 3839, 3840, 3841, 100_000, 2_000_003])
def test_sort_exact(k, cuda_dev):
    rng = np.random.default_rng(k)
    tiles = rng.integers(0, 8160, k).astype(np.uint64)
    depth = rng.uniform(0.2, 60, k).astype(np.float32).view(np.uint32).astype(np.uint64)
    if k > 10:
        depth[::5] = depth[1]  # ties keep input order
    keys = (tiles << np.uint64(32)) | depth
    vals = rng.permutation(k).astype(np.uint32)
    sk, sv = fg.sort_keys(torch.from_numpy(keys).to(cuda_dev), torch.from_numpy(vals).to(cuda_dev),
                          num_tiles=8160)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(sk.cpu().numpy(), keys[order])
    assert np.array_equal(sv.cpu().numpy(), vals[order])


def test_sort_full_64bit(cuda_dev):
    rng = np.random.default_rng(77)
    k = 300_000
    keys = rng.integers(0, 2 ** 63, k, dtype=np.int64).astype(np.uint64) * np.uint64(2)
    vals = np.arange(k, dtype=np.uint32)
    sk, sv = fg.sort_keys(torch.from_numpy(keys).to(cuda_dev), torch.from_numpy(vals).to(cuda_dev),
                          key_bits=64)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(sk.cpu().numpy(), keys[order]) and np.array_equal(sv.cpu().numpy(), vals[order])


def test_tile_order_heaviest_first(cuda_dev):
    """fgs_tile_order: a permutation of the tiles whose count class
    ceil(count/16) (capped at 255) never increases along the order."""
    import ctypes as C

    from fastgs_core_b200._lib import lib

    rng = np.random.default_rng(7)
    T = 5003
    counts = rng.integers(0, 5000, T).astype(np.int64)
    counts[rng.random(T) < 0.3] = 0
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    ranges = np.stack([starts, starts + counts], 1).astype(np.uint32)
    r = torch.from_numpy(ranges.view(np.int32)).to(cuda_dev)
    order = torch.empty(T, dtype=torch.int32, device=cuda_dev)
    assert lib().fgs_tile_order(T, C.c_void_p(r.data_ptr()), C.c_void_p(order.data_ptr()), None) == 0
    torch.cuda.synchronize()
    o = order.cpu().numpy()
    assert np.array_equal(np.sort(o), np.arange(T))
    cls = np.minimum((counts[o] + 15) // 16, 255)
    assert np.all(np.diff(cls) <= 0)


@pytest.mark.parametrize("case", CASES[1:4], ids=[f"c{c[0]}" for c in CASES[1:4]])
def test_rasterize_backward_recompute_path(case, cuda_dev):
    """The functional rasterize_backward (no contribution mask from the
    forward pass: every pair re-decided, exact exponential) against the
    oracle's rasterize-level gradients. The autograd path of the chain tests
    covers the masked variant."""
    seed, n, deg, W, H, ls, om, bg = case
    scene, cam = S.small_scene(seed, n, deg, W, H, log_scale_mu=ls, op_mu=om)
    ins = S.render_inputs(scene, cam, bg)
    cot = np.random.default_rng(seed + 100).normal(size=(3, W * H)).astype(np.float32)
    f, b = _oracle(ins, W, H, cam, deg, cot)
    res, _ = run_chain(ins, W, H, cam.tan_fovx, cam.tan_fovy, deg, cuda_dev)
    T = res["ranges"].shape[0]
    fo = {"bucket_to_tile": res["sample_bucket_to_tile"], "sampled_t": res["sample_t"],
          "sampled_ar": res["sample_ar"], "final_t": res["img_final_t"],
          "n_contrib": res["img_n_contrib"], "max_contrib": res["img_max_contrib"],
          "pixel_colors": res["img_pixel_colors"]}
    fo = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda_dev) for k, v in fo.items()}
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev)  # noqa: E731
    g = fg.rasterize_backward(d(res["ranges"]), d(res["point_list"]), d(res["bucket_offsets"]),
                              d(res["geom_means2d"]), d(res["geom_rgb"]), d(res["geom_conic_opacity"]),
                              d(np.asarray(bg, np.float32)), d(cot), fo, W, H, T, res["num_buckets"])
    for mine, theirs in (("d_means2d", "dmeans2d"), ("d_colors", "dcolors"),
                         ("d_conic_opacity", "dconic_opacity"), ("d_viewspace_points", "dviewspace_raster")):
        got = g[mine].cpu().numpy().reshape(b[theirs].shape)
        assert rel_err(got, b[theirs]) < GRAD_TOL, (mine, rel_err(got, b[theirs]))


def test_tile_prep_ordered_matches_parts(cuda_dev):
    """fgs_tile_prep_ordered = fgs_tile_prep + fgs_tile_order + invalidating
    bucket_to_tile past the bucket total."""
    import ctypes as C

    from fastgs_core_b200._lib import lib

    rng = np.random.default_rng(11)
    T = 1900
    tiles = np.sort(rng.integers(0, T, 50_000)).astype(np.uint64)
    keys = (tiles << np.uint64(32)) | rng.integers(0, 2**31, tiles.size).astype(np.uint64)
    k = torch.from_numpy(keys.view(np.int64)).to(cuda_dev)
    K = keys.size
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    outs = []
    for ordered in (False, True):
        ranges = torch.empty(2 * T, dtype=torch.int32, device=cuda_dev)
        bc = torch.empty(T, dtype=torch.int32, device=cuda_dev)
        bo = torch.empty(T, dtype=torch.int32, device=cuda_dev)
        bs = torch.empty(1, dtype=torch.int64, device=cuda_dev)
        order = torch.empty(T, dtype=torch.int32, device=cuda_dev)
        blen = K // 32 + T
        b2t = torch.full((blen,), 7, dtype=torch.int32, device=cuda_dev)
        if ordered:
            assert lib().fgs_tile_prep_ordered(K, T, p(k), p(ranges), p(bc), p(bo), p(bs), p(order),
                                               p(b2t), blen, None) == 0
        else:
            assert lib().fgs_tile_prep(K, T, p(k), p(ranges), p(bc), p(bo), p(bs), None) == 0
            assert lib().fgs_tile_order(T, p(ranges), p(order), None) == 0
        torch.cuda.synchronize()
        outs.append((ranges.cpu().numpy(), bc.cpu().numpy(), bo.cpu().numpy(), int(bs.item()),
                     order.cpu().numpy(), b2t.cpu().numpy()))
    (r1, c1, o1, s1, ord1, _), (r2, c2, o2, s2, ord2, b2t) = outs
    assert np.array_equal(r1, r2) and np.array_equal(c1, c2) and np.array_equal(o1, o2) and s1 == s2
    counts = r2[1::2].astype(np.int64) - r2[0::2]
    assert np.array_equal(np.sort(ord2), np.arange(T))
    cls = np.minimum((counts[ord2] + 15) // 16, 255)
    assert np.all(np.diff(cls) <= 0)
    assert np.all(b2t[:s2] == 7) and np.all(b2t[s2:] == -1)
