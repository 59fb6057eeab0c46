"""The data-parallel host logic on CPU ranks (gloo, world size 2): view
sharding and the step-buffer reduction the GPU step runs over NCCL."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastgs_core_b200.train import (FLOATS_PER_GAUSSIAN, STATS_SUM, allreduce_step, fold_stats,
                                    local_views)


def test_local_views():
    assert local_views(8, 1, 0) == list(range(8))
    assert local_views(8, 2, 1) == [1, 3, 5, 7]
    assert local_views(3, 4, 3) == []
    allv = sorted(v for r in range(3) for v in local_views(8, 3, r))
    assert allv == list(range(8))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(rank)
    buf = torch.randn((FLOATS_PER_GAUSSIAN + STATS_SUM + 1) * n, generator=g)
    mine = buf.clone()
    allreduce_step(buf, n)
    stats = torch.ones(4 * n)
    fold_stats(stats, buf[FLOATS_PER_GAUSSIAN * n:], n)
    q.put((rank, mine, buf, stats))
    dist.barrier()
    dist.destroy_process_group()


def test_allreduce_step_gloo():
    n, world = 5, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (m, b, s)) for r, m, b, s in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    split = (FLOATS_PER_GAUSSIAN + STATS_SUM) * n
    total = res[0][0] + res[1][0]
    mx = torch.maximum(res[0][0], res[1][0])
    for r in range(world):
        b = res[r][1]
        assert torch.allclose(b[:split], total[:split])
        assert torch.equal(b[split:], mx[split:])
        s = res[r][2]
        assert torch.allclose(s[:3 * n], 1 + total[FLOATS_PER_GAUSSIAN * n:split])
        assert torch.equal(s[3 * n:], torch.maximum(torch.ones(n), mx[split:]))
