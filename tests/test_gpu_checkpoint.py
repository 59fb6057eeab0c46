"""Checkpoint / resume of the training driver, and run-to-run determinism of
the binning and the rendered image (GPU)."""
import numpy as np
import pytest
import torch

from fastgs_core_b200 import synthetic as S
from fastgs_core_b200.policy import DriverConfig, FastGSDriver
from fastgs_core_b200.train import Trainer

pytestmark = pytest.mark.gpu


def _setup(dev):
    scene, cam = S.small_scene(21, 2500, 3, 80, 64, log_scale_mu=-3.0)
    cams = [cam] + [S.look_at_camera((0.5 * k, 0.3, 4.0), (0, 0, 0), 80, 64, 55.0) for k in range(1, 4)]
    g = torch.Generator().manual_seed(11)
    targets = [torch.rand(3 * 80 * 64, generator=g).to(dev) for _ in cams]
    return scene, cams, targets


def _cfg():
    return DriverConfig(mse_until=2, densify_until_step=0, final_prune_start=10 ** 9,
                        sh_degree_interval=2)


def test_driver_resume_continues_the_run(cuda_dev, tmp_path):
    scene, cams, targets = _setup(cuda_dev)
    # eps = 1 keeps Adam linear in the gradient, so the float-atomic noise of
    # two runs stays at the noise level
    drv = FastGSDriver(Trainer(scene, cuda_dev, eps=1.0), cams, targets, _cfg(), seed=5)
    for _ in range(4):
        drv.step()
    path = tmp_path / "ckpt.pt"
    torch.save(drv.state_dict(), path)
    saved = torch.load(path, weights_only=False)
    views_a = [drv.step()["view"] for _ in range(3)]
    want = drv.tr.params.cpu()

    other, _ = S.small_scene(99, 10, 3, 80, 64)  # any starting point: the checkpoint replaces it
    drv2 = FastGSDriver(Trainer(other, cuda_dev, eps=1.0), cams, targets, _cfg(), seed=123)
    drv2.load_state_dict(saved)
    tr2 = drv2.tr
    assert tr2.n == saved["trainer"]["n"] and tr2.step_count == saved["trainer"]["step_count"]
    assert torch.equal(tr2.params.cpu(), saved["trainer"]["params"])
    m, v = tr2.full_moments()
    assert torch.equal(m.cpu(), saved["trainer"]["exp_avg"]) and torch.equal(v.cpu(), saved["trainer"]["exp_avg_sq"])
    assert torch.equal(tr2.stats.cpu(), saved["trainer"]["stats"])
    views_b = [drv2.step()["view"] for _ in range(3)]
    assert views_a == views_b  # the generator resumed where it was
    got = tr2.params.cpu()
    assert float((got - want).abs().max()) <= 1e-5 * float(want.abs().max())


def test_binning_and_image_are_deterministic(cuda_dev):
    scene, cams, _ = _setup(cuda_dev)
    tr = Trainer(scene, cuda_dev)
    tr.activate()
    out = []
    for _ in range(2):
        img = tr.render_view(cams[1]).clone()
        k, v = (t.clone() for t in tr.last_sorted)
        out.append((img, k, v, tr.ws.b["ncontrib"][:80 * 64].clone(), tr.ws.b["ranges"][:2 * 20].clone()))
    for a, b in zip(*out):
        assert torch.equal(a, b)
