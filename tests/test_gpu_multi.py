"""Data-parallel training on 2 GPUs (skipped with fewer), against one process
that renders both views itself:

* one step at the real Adam epsilon (1e-8), every exchange (the NVLink
  multicast kernel fgs_adam_step_multicast, the peer kernel
  fgs_adam_step_peers, the push exchange fgs_preprocess_backward_push +
  fgs_adam_step_owner, the copy-engine pipeline around fgs_adam_step_gathered, and NCCL reduce-scatter / all-gather): the Adam moments agree within the float-atomic noise of the
  gradients; the parameter update agrees where the gradient stands out of
  that noise (elsewhere Adam's normalised step of a near-zero gradient takes
  either sign, and the test bounds it by the learning rate); the
  densification statistics agree;
* densification in the middle of a run: steps, densify_and_prune_fastgs on
  the all-reduced statistics with the same scores and generator on every
  rank, then more steps on the new set of Gaussians; the replicas stay
  identical and follow the single process. Also with the SH part of the
  exchange overlapped with the next render's geometry (FGS_OVERLAP_EXCHANGE).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

LR = {"means": 3e-3, "dc": 1e-3, "rest": 1e-3 / 20.0, "opacity": 1e-3, "scales": 1e-3,
      "rotations": 1e-3}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(seed=41):
    from fastgs_core_b200 import synthetic as S

    scene, cam0 = S.small_scene(seed, 3000, 3, 96, 64, log_scale_mu=-3.0)
    rng = np.random.default_rng(seed)
    cams = S.orbit_cameras(rng, 2, 4.0, 0.5, 96, 64, 55.0)
    tg = [np.random.default_rng(seed + k).uniform(0, 1, 3 * 96 * 64).astype(np.float32) for k in range(2)]
    return scene, cams, tg


def _densify_inputs(n):
    rng = np.random.default_rng(5)
    importance = np.where(rng.random(n) < 0.5, 10.0, 1.0).astype(np.float32)
    pruning = rng.uniform(0, 0.99, n).astype(np.float32)
    return importance, pruning


def _densify_args():
    from fastgs_core_b200 import densify as D

    # thresholds low enough that the two steps' statistics clone and split
    return D.DensifyArgs(grad_thresh=1e-6, grad_abs_thresh=1e-6, min_opacity=0.02)


def _run(tr, cams, targets, mode):
    """The sequence both the ranks and the single process run."""
    from fastgs_core_b200 import densify as D

    if mode == "step":
        tr.step(cams, targets)
        return None
    for _ in range(2):
        tr.step(cams, targets)
    imp, pruning = _densify_inputs(tr.n)
    # scene extent 5: dense bound 0.05 sits inside the log-scale spread (clones and splits)
    res = D.densify_and_prune_fastgs(tr, _densify_args(), 5.0, imp, pruning, np.random.default_rng(9))
    tr.step(cams, targets)
    return res


def _snapshot(tr):
    m, v = tr.full_moments()
    return (tr.comm, tr.n, tr.params.cpu(), m.cpu(), v.cpu(), tr.global_stats().cpu())


def _worker(rank, port, comm, mode, eps, q):
    import torch.distributed as dist

    from fastgs_core_b200.train import Trainer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_DEBUG="WARN")
    # "<comm>+overlap": the SH exchange overlapped with the next render's geometry
    comm, _, ov = comm.partition("+")
    os.environ["FGS_OVERLAP_EXCHANGE"] = "1" if ov == "overlap" else "0"
    freeze = ov == "freeze"  # "<comm>+freeze": the SH rest group does not step
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        scene, cams, tg = _setup()
        tr = Trainer(scene, dev, process_group=dist.group.WORLD, comm=comm, eps=eps)
        if freeze:
            tr.lrs.rest = -1.0
        targets = [torch.from_numpy(t).to(dev) if k == rank else None for k, t in enumerate(tg)]
        res = _run(tr, cams, targets, mode)
        torch.cuda.synchronize()
        q.put((rank, res) + _snapshot(tr))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _spawn(comm, mode, eps):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, comm, mode, eps, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        item = q.get(timeout=600)
        out[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


def _single(mode, eps, freeze=False):
    from fastgs_core_b200.train import Trainer

    scene, cams, tg = _setup()
    dev = torch.device("cuda", 0)
    tr = Trainer(scene, dev, eps=eps)
    if freeze:
        tr.lrs.rest = -1.0
    targets = [torch.from_numpy(t).to(dev) for t in tg]
    res = _run(tr, cams, targets, mode)
    torch.cuda.synchronize()
    return tr, res, _snapshot(tr)


def _lr_vector(n):
    lr = torch.empty(59 * n)
    for (a, b), r in zip(((0, 3), (3, 6), (6, 51), (51, 52), (52, 55), (55, 59)), LR.values()):
        lr[a * n:b * n] = r
    return lr


def _rel(a, b):
    return float((a - b).abs().max() / max(float(b.abs().max()), 1e-30))


@pytest.mark.parametrize("comm", ["multicast", "p2p", "push", "ce", "nccl"])
def test_two_rank_step_matches_single_process(comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(comm, "step", 1e-8)
    if comm != "nccl" and res[0][1] != comm:
        pytest.skip("symmetric memory (NVLink multicast / peer mappings) unavailable on this box")
    assert res[0][1] == comm
    tr, _, (_, n, want_p, want_m, want_v, want_s) = _single("step", 1e-8)
    g = tr.grads.cpu()
    p0 = torch.from_numpy(np.concatenate([getattr(_setup()[0], k).ravel() for k in (
        "means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations")]))
    lr = _lr_vector(n)
    # the gradient stands out of the atomic-order noise
    big = g.abs() > 1e-4 * g.abs().max()
    for r in range(2):
        _, _, _, p, m, v, s = res[r]
        assert _rel(m, want_m) < 1e-5, (r, _rel(m, want_m))
        assert _rel(v, want_v) < 1e-5, (r, _rel(v, want_v))
        step, want_step = p - p0, want_p - p0
        assert bool(((step - want_step).abs()[big] <= 1e-3 * lr[big]).all()), r
        assert bool((step.abs() <= lr * (1 + 1e-5)).all()), r
        assert _rel(s, want_s) < 1e-4, r
    assert torch.equal(res[0][3], res[1][3])  # replicas agree exactly
    assert big.float().mean() > 0.3


@pytest.mark.parametrize("comm", ["multicast", "p2p", "push", "ce", "nccl", "multicast+overlap",
                                  "p2p+overlap"])
def test_two_rank_densify_matches_single_process(comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    # eps = 1: Adam's update is linear in the gradient, so the two runs' float
    # noise does not grow into different sign decisions over the steps
    res = _spawn(comm, "densify", 1.0)
    if comm != "nccl" and res[0][1] != comm.partition("+")[0]:
        pytest.skip("symmetric memory (NVLink multicast / peer mappings) unavailable on this box")
    _, want_res, (_, n, want_p, want_m, want_v, want_s) = _single("densify", 1.0)
    assert want_res["cloned"] > 0 and want_res["split_sources"] > 0
    for r in range(2):
        got_res, _, rn, p, m, v, s = res[r]
        assert got_res == want_res, r
        assert rn == n
        assert _rel(p, want_p) < 1e-5, (r, _rel(p, want_p))
        assert _rel(m, want_m) < 1e-3 and _rel(v, want_v) < 1e-3, r
        assert _rel(s, want_s) < 1e-3, r
    assert torch.equal(res[0][3], res[1][3])  # replicas agree exactly


@pytest.mark.parametrize("comm", ["multicast", "p2p"])
def test_two_rank_step_with_frozen_sh_group(comm):
    """A step in which the SH rest group does not step (the reference's
    cadence): the exchange moves only the other parts of the shard; the SH
    coefficients and their moments stay as they were, the rest follows the
    single process."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(comm + "+freeze", "step", 1.0)
    if res[0][1] != comm:
        pytest.skip("symmetric memory (NVLink multicast / peer mappings) unavailable on this box")
    _, _, (_, n, want_p, want_m, want_v, _) = _single("step", 1.0, freeze=True)
    scene = _setup()[0]
    p0 = torch.from_numpy(np.concatenate([getattr(scene, k).ravel() for k in (
        "means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations")]))
    for r in range(2):
        _, _, _, p, m, v, _ = res[r]
        assert torch.equal(p[6 * n:51 * n], p0[6 * n:51 * n]), r
        assert not bool(m[6 * n:51 * n].any()) and not bool(v[6 * n:51 * n].any()), r
        assert _rel(p, want_p) < 1e-5, (r, _rel(p, want_p))
        assert _rel(m, want_m) < 1e-4 and _rel(v, want_v) < 1e-4, r
    assert torch.equal(res[0][3], res[1][3])
