"""GPU tests of the training-step kernels against plain torch fp32
references of the same operations."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import fastgs_core_b200 as fg
from fastgs_core_b200 import _lib, synthetic as S
from fastgs_core_b200.train import Trainer
from tests._gpu_util import rel_err

pytestmark = pytest.mark.gpu


def _p(t):
    import ctypes as C
    return C.c_void_p(t.data_ptr())


def _stream():
    import ctypes as C
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def torch_l1_dssim(img, tgt, w_l1=1.0, w_ssim=0.2):
    """fp32 torch reference: 11x11 Gaussian window (sigma 1.5), zero padding."""
    g = torch.exp(-((torch.arange(11, dtype=torch.float32, device=img.device) - 5) ** 2) / (2 * 1.5 ** 2))
    g = g / g.sum()
    w = (g[:, None] * g[None, :]).expand(3, 1, 11, 11).contiguous()
    x, y = img[None], tgt[None]
    conv = lambda t: F.conv2d(t, w, padding=5, groups=3)  # noqa: E731
    mx, my = conv(x), conv(y)
    sxx, syy, sxy = conv(x * x) - mx * mx, conv(y * y) - my * my, conv(x * y) - mx * my
    C1, C2 = 0.01 ** 2, 0.03 ** 2
    s = ((2 * mx * my + C1) * (2 * sxy + C2)) / ((mx * mx + my * my + C1) * (sxx + syy + C2))
    return w_l1 * (x - y).abs().mean() + w_ssim * (1 - s.mean())


@pytest.mark.parametrize("W,H", [(64, 48), (100, 37), (1920, 1080)])
def test_l1_dssim_loss(W, H, cuda_dev):
    g = torch.Generator(device="cpu").manual_seed(W)
    img = torch.rand((3, H, W), generator=g).to(cuda_dev)
    tgt = torch.rand((3, H, W), generator=g).to(cuda_dev)
    L = _lib.lib()
    scr = torch.empty(int(L.fgs_loss_scratch_bytes(W, H)) // 4 + 1, device=cuda_dev)
    out = torch.empty(3, device=cuda_dev)
    dimg = torch.empty_like(img)
    _lib.check(L.fgs_l1_dssim_loss(W, H, _p(img), _p(tgt), 1.0, 0.2, _p(out), _p(dimg), _p(scr),
                                   _stream()), "loss")
    x = img.clone().requires_grad_(True)
    ref = torch_l1_dssim(x, tgt)
    ref.backward()
    assert abs(out[0].item() - ref.item()) < 1e-5 * max(1.0, abs(ref.item()))
    assert rel_err(dimg.cpu().numpy(), x.grad.cpu().numpy()) < 1e-4


def test_adam_groups(cuda_dev):
    n = 1001
    total = 59 * n
    g = torch.Generator().manual_seed(0)
    p = torch.randn(total, generator=g).to(cuda_dev)
    gr = torch.randn(total, generator=g).to(cuda_dev)
    m = torch.randn(total, generator=g).abs().to(cuda_dev)
    v = torch.randn(total, generator=g).abs().to(cuda_dev)
    ends = np.array([3, 6, 51, 52, 55, 59]) * n
    lrs = [3e-3, 1e-3, 5e-5, 1e-3, 1e-3, 2e-3]
    lr = torch.empty(total, device=cuda_dev)
    lo = 0
    for e, r in zip(ends, lrs):
        lr[lo:e] = r
        lo = e
    import ctypes as C
    for bc, step in ((0, 1), (1, 7)):
        p0, m0, v0 = p.clone(), m.clone(), v.clone()
        _lib.check(_lib.lib().fgs_adam_step(total, _p(p), _p(gr), _p(m), _p(v), 6,
                                            (C.c_int64 * 6)(*ends.tolist()), (C.c_float * 6)(*lrs),
                                            0.9, 0.99, 1e-8, step, bc, _stream()), "adam")
        m1 = 0.9 * m0 + 0.1 * gr
        v1 = 0.99 * v0 + 0.01 * gr * gr
        mh, vh = (m1 / (1 - 0.9 ** step), v1 / (1 - 0.99 ** step)) if bc else (m1, v1)
        p1 = p0 - lr * mh / (vh.sqrt() + 1e-8)
        assert torch.allclose(m, m1, rtol=1e-6, atol=1e-7)
        assert torch.allclose(v, v1, rtol=1e-6, atol=1e-7)
        assert torch.allclose(p, p1, rtol=1e-5, atol=1e-6)


def _api_reference_grads(scene, cam, target, dev):
    """Raw-parameter gradients through the public API + torch activations +
    the torch loss reference (what the fused training path must reproduce)."""
    raw = {k: torch.from_numpy(np.ascontiguousarray(getattr(scene, k))).to(dev).requires_grad_(True)
           for k in ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales",
                     "rotations")}
    vs = torch.zeros((scene.n, 4), device=dev, requires_grad=True)
    ins = dict(means3d=raw["means3d"], dc=raw["features_dc"], sh=raw["features_rest"],
               opacities=torch.sigmoid(raw["opacity_logits"]), scales=torch.exp(raw["log_scales"]),
               rotations=raw["rotations"] / (raw["rotations"].norm(dim=1, keepdim=True) + 1e-8),
               viewmatrix=torch.from_numpy(cam.viewmatrix).to(dev),
               projmatrix=torch.from_numpy(cam.projmatrix).to(dev),
               campos=torch.from_numpy(cam.campos).to(dev), background=torch.zeros(3, device=dev),
               metric_map=torch.zeros(cam.width * cam.height, dtype=torch.int32, device=dev),
               viewspace_points=vs)
    out = fg.rasterize_gaussians(ins, cam.width, cam.height, 16, 16, cam.tan_fovx, cam.tan_fovy, 3)
    img = out["out_color"].view(3, cam.height, cam.width)
    loss = torch_l1_dssim(img, target.view(3, cam.height, cam.width))
    loss.backward()
    return {k: v.grad for k, v in raw.items()}, vs.grad, out["radii"], loss.item()


def test_training_view_matches_api_autograd(cuda_dev):
    scene, cam = S.small_scene(31, 3000, 3, 96, 64, log_scale_mu=-3.0)
    target = torch.rand(3 * cam.width * cam.height, generator=torch.Generator().manual_seed(3)).to(cuda_dev)
    want, dvs, radii, loss_ref = _api_reference_grads(scene, cam, target, cuda_dev)
    tr = Trainer(scene, cuda_dev)
    tr.activate()
    tr.step_stats.zero_()
    lo = torch.zeros(4, device=cuda_dev)
    tr.render_view(cam, target, accumulate=False, loss_out=lo)
    assert abs(lo[0].item() - loss_ref) < 1e-5
    for k, g in want.items():
        got = tr.grad_view(k)
        assert rel_err(got.cpu().numpy(), g.cpu().numpy()) < 1e-3, k
    # densification statistics of this view
    n = scene.n
    vis = (radii > 0)
    st = tr.step_stats
    exp_acc = torch.where(vis, dvs[:, :2].norm(dim=1), torch.zeros_like(dvs[:, 0]))
    exp_abs = torch.where(vis, dvs[:, 2:].norm(dim=1), torch.zeros_like(dvs[:, 0]))
    assert rel_err(st[:n].cpu().numpy(), exp_acc.cpu().numpy()) < 1e-3
    assert rel_err(st[n:2 * n].cpu().numpy(), exp_abs.cpu().numpy()) < 1e-3
    assert torch.equal(st[2 * n:3 * n], vis.float())
    assert torch.equal(st[3 * n:], torch.where(vis, radii.float(), torch.zeros_like(st[3 * n:])))
    # a second view accumulates
    g1 = tr.grads.clone()
    tr.render_view(cam, target, accumulate=True, loss_out=lo)
    assert rel_err(tr.grads.cpu().numpy(), (2 * g1).cpu().numpy()) < 1e-3


def test_trainer_step_applies_adam(cuda_dev):
    scene, cam = S.small_scene(32, 2000, 3, 64, 64)
    target = torch.rand(3 * 64 * 64, generator=torch.Generator().manual_seed(4)).to(cuda_dev)
    tr = Trainer(scene, cuda_dev)
    tr.fuse_adam = False  # the separate Adam launch, which leaves the gradient readable
    p0 = tr.params.clone()
    lo = torch.zeros(4, device=cuda_dev)
    tr.step([cam], [target], loss_out=lo)
    g = tr.grads
    m = 0.1 * g
    v = 0.01 * g * g
    n = scene.n
    lr = torch.empty_like(p0)
    for (a, b), r in zip(((0, 3), (3, 6), (6, 51), (51, 52), (52, 55), (55, 59)),
                         (3e-3, 1e-3, 5e-5, 1e-3, 1e-3, 1e-3)):
        lr[a * n:b * n] = r
    assert torch.allclose(tr.params, p0 - lr * m / (v.sqrt() + 1e-8), rtol=1e-5, atol=1e-7)
    assert (tr.stats[2 * n:3 * n] > 0).any()
    first = lo[0].item()
    for _ in range(30):
        tr.step([cam], [target], loss_out=lo)
    assert lo[0].item() < first  # optimising the scene lowers the loss


def test_metric_map_and_scores(cuda_dev):
    P, n = 4096, 500
    g = torch.Generator().manual_seed(5)
    pred = torch.rand(3 * P, generator=g).to(cuda_dev)
    tgt = torch.rand(3 * P, generator=g).to(cuda_dev)
    L = _lib.lib()
    mm = torch.empty(P, dtype=torch.int32, device=cuda_dev)
    l1 = torch.empty(1, device=cuda_dev)
    scr = torch.empty(P + 2, device=cuda_dev)
    _lib.check(L.fgs_metric_map(P, _p(pred), _p(tgt), 0.06, _p(mm), _p(l1), _p(scr), _stream()), "mm")
    l1m = (pred.view(3, P) - tgt.view(3, P)).abs().mean(0)
    norm = (l1m - l1m.min()) / torch.clamp(l1m.max() - l1m.min(), min=1e-6)
    assert torch.equal(mm, (norm > 0.06).int())
    assert abs(l1.item() - (pred - tgt).abs().sum().item()) < 1e-2
    counts = torch.randint(0, 50, (n,), generator=g, dtype=torch.int32).to(cuda_dev)
    ca = torch.zeros(n, device=cuda_dev)
    sa = torch.zeros(n, device=cuda_dev)
    for _ in range(3):
        _lib.check(L.fgs_score_accumulate(n, _p(counts), _p(l1), 3 * P, _p(ca), _p(sa), _stream()), "acc")
    imp = torch.empty(n, device=cuda_dev)
    pr = torch.empty(n, device=cuda_dev)
    s2 = torch.empty(2, dtype=torch.int32, device=cuda_dev)
    _lib.check(L.fgs_score_finalize(n, _p(ca), _p(sa), 3, _p(imp), _p(pr), _p(s2), _stream()), "fin")
    photometric = l1.item() / (3 * P)
    assert torch.equal(imp, torch.floor(ca / 3))
    want = sa.cpu().numpy()
    want = (want - want.min()) / max(want.max() - want.min(), 1e-6)
    np.testing.assert_allclose(pr.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    assert np.allclose(sa.cpu().numpy(), 3 * photometric * counts.float().cpu().numpy(), rtol=1e-5)


def test_adam_fused_into_backward_matches_separate(cuda_dev):
    """fgs_preprocess_backward_adam equals fgs_preprocess_backward_train +
    fgs_adam_step bit for bit on the same inputs (n not a multiple of 4: the
    attribute segments of the flat buffer are not 16-byte aligned)."""
    import ctypes as C

    from fastgs_core_b200._lib import PreprocessParams, lib

    scene, cam = S.small_scene(33, 2003, 3, 80, 48)
    n = scene.n
    target = torch.rand(3 * 80 * 48, generator=torch.Generator().manual_seed(5)).to(cuda_dev)
    tr = Trainer(scene, cuda_dev, bias_correction=True)
    tr.fuse_adam = False
    tr.step([cam], [target])  # non-zero moments
    tr.activate()
    tr.render_view(cam, target)  # leaves this view's backward inputs in the workspace
    torch.cuda.synchronize()
    ws = tr.ws.b
    cm = tr.last_cam
    gm, gc, gk, gv = tr.raster_grads
    prm = PreprocessParams(n, 3, 15, 1.0, 1.0, float(cam.tan_fovx), float(cam.tan_fovy), 80, 48, 0, 0)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    lrs = (C.c_float * 6)(3e-3, 1e-3, 5e-5, 1e-2, 5e-3, 1e-3)
    total = 59 * n
    P1, P2 = tr.params.clone(), tr.params.clone()
    M1, M2 = tr.exp_avg[:total].clone(), tr.exp_avg[:total].clone()
    V1, V2 = tr.exp_avg_sq[:total].clone(), tr.exp_avg_sq[:total].clone()
    G = torch.empty(total, device=cuda_dev)
    st1, st2 = torch.zeros(4 * n, device=cuda_dev), torch.zeros(4 * n, device=cuda_dev)
    L = lib()
    cams = [p(cm[0:16]), p(cm[16:32]), p(cm[32:35])]
    assert L.fgs_preprocess_backward_train(
        C.byref(prm), p(P1), *cams, p(ws["cov3d"]), p(gc), p(gm), p(gk), p(gv), p(ws["radii"]),
        p(ws["clamped"]), 0, p(G), p(st1), None) == 0
    ends = (C.c_int64 * 6)(*[k * n for k in (3, 6, 51, 52, 55, 59)])
    assert L.fgs_adam_step(total, p(P1), p(G), p(M1), p(V1), 6, ends, lrs, 0.9, 0.99, 1e-8, 2, 1,
                           None) == 0
    assert L.fgs_preprocess_backward_adam(
        C.byref(prm), *cams, p(ws["cov3d"]), p(gc), p(gm), p(gk), p(gv), p(ws["radii"]),
        p(ws["clamped"]), p(P2), p(M2), p(V2), lrs, 0.9, 0.99, 1e-8, 2, 1, p(st2), None) == 0
    torch.cuda.synchronize()
    assert not torch.equal(P1, tr.params)
    assert torch.equal(P1, P2)
    assert torch.equal(M1, M2)
    assert torch.equal(V1, V2)
    assert torch.equal(st1, st2)


def test_trainer_fused_adam_step(cuda_dev):
    """The trainer's one-view step with Adam fused into the backward pass
    follows the separate path (within the float-atomic noise of the raster
    backward; eps = 1 keeps Adam from amplifying it)."""
    scene, cam = S.small_scene(34, 1999, 3, 64, 64)
    target = torch.rand(3 * 64 * 64, generator=torch.Generator().manual_seed(6)).to(cuda_dev)
    trs = [Trainer(scene, cuda_dev, eps=1.0), Trainer(scene, cuda_dev, eps=1.0)]
    trs[1].fuse_adam = False
    p0 = trs[0].params.clone()
    for tr in trs:
        for _ in range(3):
            tr.step([cam], [target])
    torch.cuda.synchronize()
    a, b = trs
    assert a.step_count == b.step_count == 3
    assert rel_err((a.params - p0).cpu().numpy(), (b.params - p0).cpu().numpy()) < 1e-3
    assert rel_err(a.stats.cpu().numpy(), b.stats.cpu().numpy()) < 1e-3


@pytest.mark.parametrize("n", [3000, 20_001])
def test_depth_first_binning_matches_full_sort(n, cuda_dev):
    """Depth-first binning (order Gaussians by depth, emit keys in that order,
    sort the tile bits only) gives the sorted keys and values of the full
    64-bit sort of index-order keys, bit for bit, and so the same image."""
    scene, cam = S.small_scene(40 + n % 7, n, 3, 160, 96, log_scale_mu=-3.0)
    out = []
    for depth_first in (True, False):
        tr = Trainer(scene, cuda_dev)
        tr.depth_first = depth_first
        tr.activate()
        img = tr.render_view(cam).clone()
        k, v = tr.last_sorted
        out.append((k.clone(), v.clone(), img))
    (k1, v1, i1), (k2, v2, i2) = out
    assert k1.numel() > 0
    assert torch.equal(k1, k2)
    assert torch.equal(v1, v2)
    assert torch.equal(i1, i2)


@pytest.mark.parametrize("mask", [True, False])
def test_sparse_samples_same_gradients(mask, cuda_dev):
    """Sparse bucket samples (no writes or reads for pixels that terminated
    before a bucket) give the same image and, within the atomic-order noise,
    the same gradients as the fully written layout, with and without the
    contribution mask."""
    scene, cam = S.small_scene(41, 20_000, 3, 160, 128, log_scale_mu=-2.6, op_mu=1.5)
    target = torch.rand(3 * 160 * 128, generator=torch.Generator().manual_seed(9)).to(cuda_dev)
    out = []
    for sparse in (True, False):
        tr = Trainer(scene, cuda_dev)
        tr.contrib_mask = mask
        tr.sparse_samples = sparse
        tr.activate()
        tr.step_stats.zero_()
        img = tr.render_view(cam, target).clone()
        out.append((img, tr.grads.clone(), tr.step_stats.clone()))
    (i1, g1, s1), (i2, g2, s2) = out
    assert torch.equal(i1, i2)
    assert rel_err(g1.cpu().numpy(), g2.cpu().numpy()) < 1e-5
    assert rel_err(s1.cpu().numpy(), s2.cpu().numpy()) < 1e-5


def test_l1_dssim_loss_autograd(cuda_dev):
    """fastgs_core.l1_dssim_loss as an autograd function against the torch
    fp32 reference (value and gradient)."""
    g = torch.Generator(device="cpu").manual_seed(77)
    img = torch.rand((3, 70, 90), generator=g).to(cuda_dev).requires_grad_(True)
    tgt = torch.rand((3, 70, 90), generator=g).to(cuda_dev)
    loss = fg.l1_dssim_loss(img, tgt) * 2.0
    loss.backward()
    x = img.detach().clone().requires_grad_(True)
    ref = torch_l1_dssim(x, tgt) * 2.0
    ref.backward()
    assert abs(loss.item() - ref.item()) < 1e-5 * max(1.0, abs(ref.item()))
    assert rel_err(img.grad.cpu().numpy(), x.grad.cpu().numpy()) < 1e-4


@pytest.mark.parametrize("W,H", [(64, 48), (1920, 1080)])
def test_mse_loss(W, H, cuda_dev):
    """fgs_mse_loss (the reference trainer's warm-up loss) against torch fp32."""
    g = torch.Generator(device="cpu").manual_seed(W + 1)
    img = torch.rand((3, H, W), generator=g).to(cuda_dev)
    tgt = torch.rand((3, H, W), generator=g).to(cuda_dev)
    L = _lib.lib()
    scr = torch.empty(int(L.fgs_loss_scratch_bytes(W, H)) // 4 + 1, device=cuda_dev)
    out = torch.empty(3, device=cuda_dev)
    dimg = torch.empty_like(img)
    _lib.check(L.fgs_mse_loss(W, H, _p(img), _p(tgt), 0.5, _p(out), _p(dimg), _p(scr), _stream()), "mse")
    x = img.clone().requires_grad_(True)
    ref = 0.5 * ((x - tgt) ** 2).mean()
    ref.backward()
    assert abs(out[0].item() - ref.item()) < 1e-5 * max(1.0, abs(ref.item()))
    assert abs(out[1].item() - 2 * ref.item()) < 1e-5
    assert rel_err(dimg.cpu().numpy(), x.grad.cpu().numpy()) < 1e-5


def test_driver_mse_warmup(cuda_dev):
    """FastGSDriver uses the MSE loss up to mse_until and L1 (+ D-SSIM) after."""
    from fastgs_core_b200.policy import DriverConfig, FastGSDriver

    scene, cam = S.small_scene(13, 1500, 3, 64, 48)
    target = torch.rand(3 * 64 * 48, generator=torch.Generator().manual_seed(2)).to(cuda_dev)
    tr = Trainer(scene, cuda_dev, w_ssim=0.0)
    drv = FastGSDriver(tr, [cam], [target], DriverConfig(mse_until=2, densify_until_step=0,
                                                         final_prune_start=10**9), seed=3)
    lo = torch.zeros(4, device=cuda_dev)
    modes = []
    for _ in range(4):
        drv.step(loss_out=lo)
        torch.cuda.synchronize()
        modes.append(tr.loss_mode)
        img = tr.ws.b["img"][:3 * 64 * 48]
        d = img - target
        want = (d * d).mean() if tr.loss_mode == "mse" else d.abs().mean()
        assert abs(lo[0].item() - want.item()) < 1e-4
    assert modes == ["mse", "mse", "l1_dssim", "l1_dssim"]


@pytest.mark.parametrize("degree", [0, 1, 3])
def test_split_preprocess_matches_fused(degree, cuda_dev):
    """fgs_preprocess_forward_train_geometry + fgs_preprocess_colors_train (the
    split the data-parallel trainer uses to overlap the SH exchange) give the
    outputs of the one-launch fgs_preprocess_forward_train bit for bit."""
    import ctypes as C

    scene, cam = S.small_scene(41, 3001, 3, 96, 64)
    tr = Trainer(scene, cuda_dev)
    L = _lib.lib()
    n = scene.n
    prm = _lib.PreprocessParams(n, degree, 15, 1.0, 1.0, float(cam.tan_fovx), float(cam.tan_fovy),
                                cam.width, cam.height, 0, 0)
    f = lambda: torch.from_numpy(np.concatenate([cam.viewmatrix.reshape(-1), cam.projmatrix.reshape(-1),
                                                 cam.campos.reshape(-1)]).astype(np.float32)).to(cuda_dev)
    cm = f()
    vm, pm, cp = cm[0:16], cm[16:32], cm[32:35]
    vs_in = torch.zeros(4 * n, device=cuda_dev)

    def outs():
        return dict(radii=torch.full((n,), -7, dtype=torch.int32, device=cuda_dev),
                    xys=torch.full((2 * n,), 7.0, device=cuda_dev),
                    depths=torch.full((n,), 7.0, device=cuda_dev),
                    cov3d=torch.full((6 * n,), 7.0, device=cuda_dev),
                    rgb=torch.full((3 * n,), 7.0, device=cuda_dev),
                    conic=torch.full((4 * n,), 7.0, device=cuda_dev),
                    tiles=torch.full((n,), 7, dtype=torch.uint32, device=cuda_dev),
                    clamped=torch.full((3 * n,), 7, dtype=torch.uint8, device=cuda_dev),
                    vs=torch.full((4 * n,), 7.0, device=cuda_dev))

    a, b = outs(), outs()
    s = _stream()
    assert L.fgs_preprocess_forward_train(C.byref(prm), _p(tr.params), _p(vm), _p(pm), _p(cp), _p(vs_in),
                                          _p(a["radii"]), _p(a["xys"]), _p(a["depths"]), _p(a["cov3d"]),
                                          _p(a["rgb"]), _p(a["conic"]), _p(a["tiles"]), _p(a["clamped"]),
                                          _p(a["vs"]), s) == 0
    assert L.fgs_preprocess_forward_train_geometry(C.byref(prm), _p(tr.params), _p(vm), _p(pm), _p(vs_in),
                                                   _p(b["radii"]), _p(b["xys"]), _p(b["depths"]),
                                                   _p(b["cov3d"]), _p(b["conic"]), _p(b["tiles"]),
                                                   _p(b["vs"]), s) == 0
    # geometry alone leaves the colour outputs untouched
    assert torch.all(b["rgb"] == 7.0) and torch.all(b["clamped"] == 7)
    assert L.fgs_preprocess_colors_train(C.byref(prm), _p(tr.params), _p(cp), _p(b["tiles"]),
                                         _p(b["rgb"]), _p(b["clamped"]), s) == 0
    torch.cuda.synchronize()
    assert (a["tiles"].view(torch.int32) != 0).sum().item() > 100
    for k in a:
        assert torch.equal(a[k].view(torch.uint8) if a[k].dtype != torch.uint8 else a[k],
                           b[k].view(torch.uint8) if b[k].dtype != torch.uint8 else b[k]), k
