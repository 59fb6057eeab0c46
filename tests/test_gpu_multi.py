"""Data-parallel training step on 2 GPUs (skipped with fewer): the NVLink
multicast exchange (fgs_adam_step_multicast) and the NCCL reduce-scatter /
all-gather exchange must both give the parameters and densification
statistics of one process that renders both views itself."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# A large Adam epsilon makes the update linear in the gradient: with the
# default 1e-8 the normalised step of a near-zero gradient flips with the
# 1e-7-level noise of the float atomics, which says nothing about the exchange.
EPS = 1.0


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


def _worker(rank, port, comm, q):
    import torch.distributed as dist

    from fastgs_core_b200.train import Trainer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_DEBUG="WARN")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        scene, cams, tg = _setup()
        tr = Trainer(scene, dev, process_group=dist.group.WORLD, comm=comm, eps=EPS)
        targets = [torch.from_numpy(t).to(dev) for t in tg]
        for _ in range(3):
            tr.step(cams, [targets[k] if k == rank else None for k in range(2)])
        torch.cuda.synchronize()
        q.put((rank, tr.comm, tr.params.cpu(), tr.global_stats().cpu()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("comm", ["multicast", "nccl"])
def test_two_rank_step_matches_single_process(comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from fastgs_core_b200.train import Trainer

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, comm, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, used, params, stats = q.get(timeout=600)
        res[r] = (used, params, stats)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if comm == "multicast" and res[0][0] != "multicast":
        pytest.skip("NVLink multicast unavailable on this box")
    assert res[0][0] == comm
    scene, cams, tg = _setup()
    dev = torch.device("cuda", 0)
    single = Trainer(scene, dev, eps=EPS)
    targets = [torch.from_numpy(t).to(dev) for t in tg]
    for _ in range(3):
        single.step(cams, targets)
    want_p = single.params.cpu()
    want_s = single.global_stats().cpu()
    for r in range(2):
        assert torch.allclose(res[r][1], want_p, rtol=1e-5, atol=1e-6), (r, (res[r][1] - want_p).abs().max())
        assert torch.allclose(res[r][2], want_s, rtol=1e-4, atol=1e-5)
    assert torch.equal(res[0][1], res[1][1])  # replicas agree exactly
    init = torch.from_numpy(np.concatenate([scene.means3d.ravel(), scene.features_dc.ravel(),
                                            scene.features_rest.ravel(), scene.opacity_logits.ravel(),
                                            scene.log_scales.ravel(), scene.rotations.ravel()]))
    assert (want_p - init).abs().max() > 1e-6  # the steps did update the parameters
