"""The data-parallel host logic on CPU ranks (gloo, world size 2 and 3): view
sharding, shard ranges, the gradient reduce-scatter, a shard-local update, the
parameter all-gather and the statistics reduction that the GPU step runs over
NCCL. The result must equal a single process applying the same update to the
summed gradients."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastgs_core_b200.train import (STATS_SUM, allgather_params, allreduce_stats, fold_stats,
                                    local_views, reduce_scatter_grads, shard_range)


def test_local_views():
    assert local_views(8, 1, 0) == list(range(8))
    assert local_views(8, 2, 1) == [1, 3, 5, 7]
    assert local_views(3, 4, 3) == []
    assert sorted(v for r in range(3) for v in local_views(8, 3, r)) == list(range(8))


def test_shard_ranges_cover_buffer():
    for total in (1, 59, 59 * 1001, 4096):
        for world in (1, 2, 3, 8):
            rs = [shard_range(total, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == total
            for (a, b), (c, d) in zip(rs, rs[1:]):
                assert b == c and a <= b
            assert all(lo % 4 == 0 for lo, hi in rs if hi > lo)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    total = 59 * n
    per = -(-total // (4 * world)) * 4
    g = torch.Generator().manual_seed(100 + rank)
    params = torch.zeros(per * world)
    params[:total] = torch.arange(total, dtype=torch.float32)  # replicated start
    grads = torch.zeros(per * world)
    grads[:total] = torch.randn(total, generator=g)
    mine = grads.clone()
    step_stats = torch.rand((STATS_SUM + 1) * n, generator=g)
    stats_in = step_stats.clone()
    shard = reduce_scatter_grads(grads, world, rank)
    lo, hi = shard_range(total, world, rank)
    params[lo:hi] -= 0.5 * shard[: hi - lo]  # shard-local update
    allgather_params(params, world, rank)
    allreduce_stats(step_stats, n)
    stats = torch.ones(4 * n)
    fold_stats(stats, step_stats, n)
    q.put((rank, mine[:total], stats_in, params[:total], stats))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_update_matches_single_process(world):
    n = 7
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: rest for r, *rest in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gsum = sum(res[r][0] for r in range(world))
    want_params = torch.arange(59 * n, dtype=torch.float32) - 0.5 * gsum
    ssum = sum(res[r][1][: STATS_SUM * n] for r in range(world))
    smax = torch.stack([res[r][1][STATS_SUM * n:] for r in range(world)]).max(0).values
    for r in range(world):
        assert torch.allclose(res[r][2], want_params, atol=1e-5)
        st = res[r][3]
        assert torch.allclose(st[: STATS_SUM * n], 1 + ssum, atol=1e-6)
        assert torch.equal(st[STATS_SUM * n:], torch.maximum(torch.ones(n), smax))


def _failing_worker(rank, world, port, q):
    """Rank 1 fails before the step's collective; rank 0 must get an error
    from the process group (its timeout or the closed connection), not hang."""
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "raised"))
        q.close()
        q.join_thread()
        os._exit(3)  # dies between steps, nothing in flight
    grads = torch.zeros(8 * world)
    try:
        reduce_scatter_grads(grads, world, rank)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error: " + type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_lost_rank_surfaces_as_an_error():
    import time

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "raised" and procs[1].exitcode == 3
    assert res[0].startswith("error"), res[0]
    assert time.time() - t0 < 100
