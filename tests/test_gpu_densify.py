"""GPU densification (fastgs_core_b200.densify) against the CPU restatement
of the reference's FastGS densification (oracle/densify_ref.py), with the
same seeded random generator on both sides. Row copies, moments and
statistics compare bit for bit; the split children's means and scales and
the capped opacity logits within 1e-5 relative (device exp/log)."""
import numpy as np
import pytest
import torch

from fastgs_core_b200 import densify as D
from fastgs_core_b200 import synthetic as S
from fastgs_core_b200.train import Trainer
from oracle import densify_ref as R

pytestmark = pytest.mark.gpu

NAMES = R.PARAMS
WIDTHS = dict(zip(NAMES, D.PARAM_WIDTHS))
SHAPES = {"means3d": (3,), "features_dc": (3,), "features_rest": (15, 3), "opacity_logits": (),
          "log_scales": (3,), "rotations": (4,)}


def split_flat(flat, n):
    out, off = {}, 0
    for k in NAMES:
        w = WIDTHS[k]
        out[k] = flat[off * n:(off + w) * n].reshape((n,) + SHAPES[k])
        off += w
    return out


def make_trainer(cuda_dev, n=3000, seed=0):
    """A trainer with random parameters, moments and statistics, kept away
    from every decision threshold (so device and host exp agree on them)."""
    rng = np.random.default_rng(seed)
    scene, _ = S.small_scene(seed, n, 3, 64, 64)
    extent = 5.0
    dense = 0.01 * extent
    big = rng.random(n) < 0.5
    scene.log_scales[:] = np.where(big[:, None], np.log(dense * rng.uniform(2, 4, (n, 3))),
                                   np.log(dense * rng.uniform(0.1, 0.5, (n, 3)))).astype(np.float32)
    low = rng.random(n) < 0.2
    scene.opacity_logits[:] = np.where(low, rng.uniform(-9, -7, n), rng.uniform(-2, 3, n)).astype(np.float32)
    tr = Trainer(scene, cuda_dev)
    total = 59 * n
    tr.exp_avg[:total] = torch.from_numpy(rng.normal(0, 1e-3, total).astype(np.float32)).to(cuda_dev)
    tr.exp_avg_sq[:total] = torch.from_numpy(rng.uniform(0, 1e-6, total).astype(np.float32)).to(cuda_dev)
    denom = rng.integers(0, 20, n).astype(np.float32)
    acc = np.where(rng.random(n) < 0.5, 1e-3, 1e-5).astype(np.float32) * np.maximum(denom, 1)
    acc_abs = np.where(rng.random(n) < 0.5, 5e-3, 1e-5).astype(np.float32) * np.maximum(denom, 1)
    maxr = np.where(rng.random(n) < 0.1, 30.0, 5.0).astype(np.float32)
    tr.stats.copy_(torch.from_numpy(np.concatenate([acc, acc_abs, denom, maxr])).to(cuda_dev))
    importance = np.where(rng.random(n) < 0.6, 10.0, 1.0).astype(np.float32)
    pruning = rng.uniform(0, 0.99, n).astype(np.float32)
    return tr, extent, importance, pruning


def oracle_state(tr, pruning=None):
    n = tr.n
    params = split_flat(tr.params.cpu().numpy(), n)
    m = split_flat(tr.exp_avg[:59 * n].cpu().numpy(), n)
    v = split_flat(tr.exp_avg_sq[:59 * n].cpu().numpy(), n)
    st = tr.stats.cpu().numpy()
    stats = {"xyz_grad_accum": st[:n], "xyz_grad_accum_abs": st[n:2 * n], "denom": st[2 * n:3 * n],
             "max_radii2d": st[3 * n:], "tmp_radii": np.zeros(n, np.float32)}
    return R.State(params, {k: (m[k], v[k]) for k in NAMES}, stats, pruning)


def compare(tr, st, approx=()):
    n = tr.n
    assert n == st.n
    got = split_flat(tr.params.cpu().numpy(), n)
    gm = split_flat(tr.exp_avg[:59 * n].cpu().numpy(), n)
    gv = split_flat(tr.exp_avg_sq[:59 * n].cpu().numpy(), n)
    for k in NAMES:
        if k in approx:
            np.testing.assert_allclose(got[k], st.params[k], rtol=1e-5, atol=1e-6, err_msg=k)
        else:
            assert np.array_equal(got[k], st.params[k]), k
        assert np.array_equal(gm[k], st.adam[k][0]), k
        assert np.array_equal(gv[k], st.adam[k][1]), k
    s = tr.stats.cpu().numpy()
    for i, k in enumerate(("xyz_grad_accum", "xyz_grad_accum_abs", "denom", "max_radii2d")):
        assert np.array_equal(s[i * n:(i + 1) * n], st.stats[k]), k


def test_prune_points(cuda_dev):
    tr, _, _, pruning = make_trainer(cuda_dev, 2001, 1)
    st = oracle_state(tr, pruning)
    mask = np.random.default_rng(5).random(tr.n) < 0.3
    R.prune_points(st, mask)
    score = D.prune_points(tr, mask, pruning)
    compare(tr, st)
    assert np.array_equal(score, st.score)


def test_clone_and_split(cuda_dev):
    tr, _, _, pruning = make_trainer(cuda_dev, 1500, 2)
    st = oracle_state(tr, pruning)
    g = np.random.default_rng(9)
    metric = g.random(tr.n) < 0.5
    clone = g.random(tr.n) < 0.3
    split = ~clone & (g.random(tr.n) < 0.5)
    c1, sc = D.densify_and_clone(tr, metric, clone, pruning)
    c2 = R.densify_and_clone(st, metric, clone)
    assert c1 == c2 > 0
    r1, r2 = np.random.default_rng(77), np.random.default_rng(77)
    a = D.densify_and_split(tr, metric, split, r1, 2, sc)
    b = R.densify_and_split(st, metric, split, r2, 2)
    assert a[:2] == b and a[0] > 0
    compare(tr, st, approx=("means3d", "log_scales"))
    assert np.array_equal(a[2], st.score)


def test_densify_and_prune_fastgs(cuda_dev):
    tr, extent, importance, pruning = make_trainer(cuda_dev, 4000, 3)
    st = oracle_state(tr, pruning)
    args = D.DensifyArgs()
    got = D.densify_and_prune_fastgs(tr, args, extent, importance, pruning, np.random.default_rng(123))
    want = R.densify_and_prune(st, args, extent, importance, np.random.default_rng(123))
    assert got == want
    assert got["cloned"] > 0 and got["split_sources"] > 0 and got["actual_removed"] > 0
    compare(tr, st, approx=("means3d", "log_scales", "opacity_logits"))
    # the trainer keeps training on the new set of Gaussians
    _, cam = S.small_scene(3, 10, 3, 64, 64)
    target = torch.rand(3 * 64 * 64, generator=torch.Generator().manual_seed(1)).to(cuda_dev)
    lo = torch.zeros(4, device=cuda_dev)
    tr.step([cam], [target], loss_out=lo)
    torch.cuda.synchronize()
    assert np.isfinite(lo[0].item())


def test_final_prune_keeps_minimum(cuda_dev):
    tr, _, _, pruning = make_trainer(cuda_dev, 500, 4)
    st = oracle_state(tr)
    got = D.final_prune_fastgs(tr, 0.5, pruning, 0.1, 300)
    want = R.final_prune(st, 0.5, pruning, 0.1, 300)
    assert got == want and got["kept"] == 300
    compare(tr, st)


def test_opacity_reset(cuda_dev):
    tr, _, _, _ = make_trainer(cuda_dev, 700, 5)
    st = oracle_state(tr)
    D.reset_opacity_logits(tr, 0.05)
    R.set_opacity_cap(st, 0.05)
    compare(tr, st, approx=("opacity_logits",))


def test_scores_fold_views(cuda_dev):
    """compute_gaussian_scores_fastgs: the metric map of each sampled view,
    the counting render and the folding, against the same steps in torch."""
    scene, cam = S.small_scene(6, 3000, 3, 96, 64, log_scale_mu=-3.0)
    cams = [cam, S.look_at_camera((0.5, 0.3, 4.0), (0, 0, 0), 96, 64, 55.0)]
    g = torch.Generator().manual_seed(8)
    P = 96 * 64
    targets = [torch.rand(3 * P, generator=g).to(cuda_dev) for _ in cams]
    tr = Trainer(scene, cuda_dev)
    imp, pr = D.compute_gaussian_scores_fastgs(tr, cams, targets, [1, 0], 0.06, True)
    n = scene.n
    counts = torch.zeros(n, device=cuda_dev)
    score = torch.zeros(n, device=cuda_dev)
    for i in (1, 0):
        pred = tr.render_view(cams[i]).clone()
        l1 = (pred.view(3, P) - targets[i].view(3, P)).abs()
        lm = l1.mean(0)
        mm = (((lm - lm.min()) / torch.clamp(lm.max() - lm.min(), min=1e-6)) > 0.06).int()
        mc = torch.empty(n, dtype=torch.int32, device=cuda_dev)
        tr.render_view(cams[i], metric_map=mm, metric_count=mc)
        counts += mc.float()
        score += l1.mean() * mc.float()
    assert counts.sum().item() > 0
    assert np.array_equal(imp, torch.floor(counts / 2).cpu().numpy())
    s = score.cpu().numpy()
    np.testing.assert_allclose(pr, (s - s.min()) / max(s.max() - s.min(), 1e-6), rtol=1e-4, atol=1e-5)


def test_driver_schedule_runs(cuda_dev):
    """FastGSDriver: the reference's loop schedule with densification, an
    opacity reset and a final prune inside a short run; frozen groups do not
    move."""
    from fastgs_core_b200.policy import DriverConfig, FastGSDriver

    scene, cam = S.small_scene(12, 4000, 3, 96, 64, log_scale_mu=-3.5)
    cams = [cam] + [S.look_at_camera((0.4 * k, 0.2, 4.0), (0, 0, 0), 96, 64, 55.0) for k in range(1, 4)]
    g = torch.Generator().manual_seed(4)
    targets = [torch.rand(3 * 96 * 64, generator=g).to(cuda_dev) for _ in cams]
    tr = Trainer(scene, cuda_dev)
    cfg = DriverConfig(sh_degree_interval=5, stage_color_steps=3, densify_from_step=4,
                       densify_until_step=30, densification_interval=8, opacity_reset_interval=20,
                       densify_camera_sample=3, final_prune_start=30, final_prune_end=50,
                       final_prune_interval=35, final_prune_min_gaussians=100)
    cfg.densify.importance_score_threshold = 0.5
    cfg.densify.grad_thresh = 1e-7
    cfg.densify.grad_abs_thresh = 1e-7
    drv = FastGSDriver(tr, cams, targets, cfg, seed=7)
    n = tr.n
    dc0 = tr.params[3 * n:6 * n].clone()
    drv.step()
    torch.cuda.synchronize()
    assert torch.equal(tr.params[3 * n:6 * n], dc0)  # colours staged out for 3 steps
    lo = torch.zeros(4, device=cuda_dev)
    outs = [drv.step(loss_out=lo) for _ in range(39)]
    torch.cuda.synchronize()
    assert np.isfinite(lo[0].item())
    dens = [o["densify"] for o in outs if "densify" in o]
    assert dens and any(d["cloned"] + d["split_sources"] > 0 for d in dens)
    assert any("opacity_reset" in o for o in outs)
    assert any("final_prune" in o for o in outs)
    assert drv.active_sh_degree == 3
    assert tr.n != n


# ---------------------------------------------------------------------------
# Against fixtures made by the reference's own densification functions
# (tests/golden/make_densify_golden.py; the CPU checker is pinned to the same
# fixtures in tests/test_densify_golden.py).
import json  # noqa: E402
import os  # noqa: E402

GOLD = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "densify_ref.npz")))


def trainer_from_fixture(cuda_dev, tag):
    z = GOLD
    p = {k: z[f"{tag}_in_{k}"] for k in NAMES}
    n = p["means3d"].shape[0]
    scene = S.Scene(p["means3d"], p["features_dc"], p["features_rest"], p["opacity_logits"],
                    p["log_scales"], p["rotations"], 3)
    tr = Trainer(scene, cuda_dev)
    m = np.concatenate([z[f"{tag}_in_m_{k}"].reshape(-1) for k in NAMES])
    v = np.concatenate([z[f"{tag}_in_v_{k}"].reshape(-1) for k in NAMES])
    tr.exp_avg[:59 * n] = torch.from_numpy(m).to(cuda_dev)
    tr.exp_avg_sq[:59 * n] = torch.from_numpy(v).to(cuda_dev)
    st = np.concatenate([z[f"{tag}_in_acc"], z[f"{tag}_in_acc_abs"], z[f"{tag}_in_denom"],
                         z[f"{tag}_in_max_radii"]])
    tr.stats.copy_(torch.from_numpy(st).to(cuda_dev))
    return tr


def compare_fixture(tr, prefix, approx=(), stats=True):
    n = tr.n
    got = split_flat(tr.params.cpu().numpy(), n)
    gm = split_flat(tr.exp_avg[:59 * n].cpu().numpy(), n)
    gv = split_flat(tr.exp_avg_sq[:59 * n].cpu().numpy(), n)
    for k in NAMES:
        want = GOLD[f"{prefix}_{k}"]
        assert got[k].shape == want.shape, k
        if k in approx:
            np.testing.assert_allclose(got[k], want, rtol=1e-5, atol=1e-6, err_msg=k)
        else:
            assert np.array_equal(got[k], want), k
        m_key = prefix.replace("_out", "_out_m").replace("_partial", "_partial_m")
        v_key = prefix.replace("_out", "_out_v").replace("_partial", "_partial_v")
        assert np.array_equal(gm[k], GOLD[f"{m_key}_{k}"]), k
        assert np.array_equal(gv[k], GOLD[f"{v_key}_{k}"]), k
    if stats:
        s = tr.stats.cpu().numpy()
        tag = prefix.split("_out")[0]
        for i, zk in enumerate(("acc", "acc_abs", "denom", "max_radii")):
            assert np.array_equal(s[i * n:(i + 1) * n], GOLD[f"{tag}_out_{zk}"]), zk


@pytest.mark.parametrize("tag", ["clone_cap", "prune_cap"])
def test_densify_and_prune_matches_reference_fixture(tag, cuda_dev):
    tr = trainer_from_fixture(cuda_dev, tag)
    args = D.DensifyArgs(**json.loads(str(GOLD[f"{tag}_args"])))
    got = D.densify_and_prune_fastgs(tr, args, float(GOLD["extent"]), GOLD[f"{tag}_in_importance"],
                                     GOLD[f"{tag}_in_pruning"],
                                     np.random.default_rng(int(GOLD[f"{tag}_seed"])))
    assert got == json.loads(str(GOLD[f"{tag}_result"]))
    compare_fixture(tr, f"{tag}_out", approx=("opacity_logits",))


def test_split_matches_reference_fixture(cuda_dev):
    """The reference's split result (recorded where its bookkeeping raises
    after the split was applied)."""
    tag = "split"
    tr = trainer_from_fixture(cuda_dev, tag)
    args = D.DensifyArgs(**json.loads(str(GOLD[f"{tag}_args"])))
    n = tr.n
    st = GOLD
    denom = np.maximum(st["split_in_denom"], 1.0)
    q_abs = np.abs(st["split_in_acc_abs"] / denom) >= args.grad_abs_thresh
    max_scale = np.max(np.exp(st["split_in_log_scales"]), axis=1)
    metric = st["split_in_importance"] > args.importance_score_threshold
    split_filter = (max_scale > args.dense * float(st["extent"])) & q_abs
    count, children, _ = D.densify_and_split(tr, metric, split_filter,
                                             np.random.default_rng(int(st["split_seed"])), 2)
    assert count > 0 and tr.n == n + count
    compare_fixture(tr, "split_partial", approx=("means3d", "log_scales"), stats=False)


def test_final_prune_reset_prune_match_reference_fixture(cuda_dev):
    tr = trainer_from_fixture(cuda_dev, "final_prune")
    got = D.final_prune_fastgs(tr, 0.5, GOLD["final_prune_in_pruning"], 0.3, 200)
    assert got == json.loads(str(GOLD["final_prune_result"]))
    compare_fixture(tr, "final_prune_out")
    tr = trainer_from_fixture(cuda_dev, "reset")
    D.reset_opacity_logits(tr, 0.05)
    compare_fixture(tr, "reset_out", approx=("opacity_logits",))
    tr = trainer_from_fixture(cuda_dev, "prune")
    D.prune_points(tr, GOLD["prune_mask"])
    compare_fixture(tr, "prune_out")
