"""Training step for FastGS on B200: view-sharded data parallelism.

One process per GPU. Every rank holds all Gaussian parameters in one flat
buffer (59 floats per Gaussian; layout in include/fastgs_b200.h). A step takes
a batch of cameras; rank r renders views r, r+R, ... through the rasterizer
kernels, back-propagates an L1 + D-SSIM loss into the flat gradient buffer
(activations fused into preprocess-backward), all-reduces the gradients and
then updates its 1/R shard of the parameters. With NVLink multicast (the
default where symmetric memory supports it) one kernel reads the rank-summed
shard gradient from the switch, runs Adam and broadcasts the new parameters
to every rank (fgs_adam_step_multicast); otherwise NCCL reduce-scatters the
gradients and all-gathers the parameter shards around a local Adam.
Densification statistics stay per rank and are combined on demand.

This is the trainer loop of scripts/train_scanner_fastgs.py:968-1019 (one
loss per view, Adam with per-group learning rates, densification statistics
from the viewspace gradient), with the render-twice defect of its loss
(:935-964, which leaves the viewspace gradient at zero) not reproduced: the
statistics come from the render the loss is taken on.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import PreprocessParams, RasterParams, check, lib
from .api import sort_key_bits, tile_grid

FLOATS_PER_GAUSSIAN = 59
STATS_SUM = 3  # grad_accum, grad_accum_abs, denom (summed across ranks)


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


@dataclass
class LearningRates:
    """Per-group learning rates (scripts/train_scanner_fastgs.py:813-817 defaults;
    SH rest uses the colour rate / 20 as OptimizerPolicyConfig.sh_lr_divisor)."""

    means: float = 3e-3
    dc: float = 1e-3
    rest: float = 1e-3 / 20.0
    opacity: float = 1e-3
    scales: float = 1e-3
    rotations: float = 1e-3


class _Grow:
    """Grow-only device buffers keyed by name."""

    def __init__(self, dev):
        self.dev = dev
        self.b: dict[str, torch.Tensor] = {}

    def get(self, name, numel, dtype):
        t = self.b.get(name)
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(max(int(numel * 1.15), 1024), dtype=dtype, device=self.dev)
            self.b[name] = t
        return t[:numel]


def _symmetric_pair(numel: int, dev, group, multicast: bool = True):
    """Parameter and gradient buffers in symmetric memory, mapped on every
    rank (peer pointers) and, with `multicast`, bound to an NVLink multicast
    object (None where that is unavailable)."""
    try:
        import torch.distributed._symmetric_memory as symm
    except ImportError:
        return None
    try:
        name = group.group_name if group is not None else "0"
        if hasattr(symm, "enable_symm_mem_for_group"):
            symm.enable_symm_mem_for_group(name)
        p = symm.empty(numel, dtype=torch.float32, device=dev)
        g = symm.empty(numel, dtype=torch.float32, device=dev)
        # zeroed before any rank can see them: with the push exchange, peers
        # add into this gradient buffer from their first backward pass on
        p.zero_()
        g.zero_()
        torch.cuda.synchronize(dev)
        hp = symm.rendezvous(p, name)
        hg = symm.rendezvous(g, name)
        if multicast and (not getattr(hp, "multicast_ptr", 0) or not getattr(hg, "multicast_ptr", 0)):
            return None
        if not multicast and len(getattr(hp, "buffer_ptrs", ())) != dist_world(group):
            return None
        return p, g, hp, hg
    except Exception:
        return None


def dist_world(group) -> int:
    import torch.distributed as dist

    return dist.get_world_size(group)


def default_comm(world: int) -> str:
    """The exchange a data-parallel step uses by default: at two ranks plain
    peer loads and stores (fgs_adam_step_peers: 118 MB per direction and
    phase at 1M Gaussians), beyond that the NVLink multicast kernel, whose
    per-GPU traffic does not grow with the number of ranks."""
    return "p2p" if world == 2 else "multicast"


def local_views(num_views: int, world: int, rank: int) -> list[int]:
    """Views of a batch this rank renders: v with v % world == rank."""
    return list(range(rank, num_views, world))


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Slice [lo, hi) of a flat buffer of ``total`` floats owned by ``rank``
    when it is padded to a multiple of 4 * world (16-byte aligned shards)."""
    per = -(-total // (4 * world)) * 4
    lo = min(total, rank * per)
    return lo, min(total, lo + per)


def reduce_scatter_grads(padded: torch.Tensor, world: int, rank: int, group=None) -> torch.Tensor:
    """Sum the per-rank gradient buffers and leave this rank its shard, in
    place (``padded`` has a 4*world-aligned length; returns the shard view)."""
    import torch.distributed as dist

    per = padded.numel() // world
    shard = padded[rank * per:(rank + 1) * per]
    dist.reduce_scatter_tensor(shard, padded, group=group)
    return shard


def allgather_params(padded: torch.Tensor, world: int, rank: int, group=None) -> None:
    """Every rank's updated parameter shard into every rank's full buffer (in place)."""
    import torch.distributed as dist

    per = padded.numel() // world
    dist.all_gather_into_tensor(padded, padded[rank * per:(rank + 1) * per], group=group)


def allreduce_stats(step_stats: torch.Tensor, n: int, group=None) -> None:
    """Sum of the 3N densification statistics, max of the N screen radii."""
    import torch.distributed as dist

    dist.all_reduce(step_stats[: STATS_SUM * n], group=group)
    dist.all_reduce(step_stats[STATS_SUM * n:STATS_SUM * n + n], op=dist.ReduceOp.MAX, group=group)


def fold_stats(stats: torch.Tensor, step_stats: torch.Tensor, n: int) -> None:
    """Running densification statistics += this step's (max for radii)."""
    stats[: STATS_SUM * n].add_(step_stats[: STATS_SUM * n])
    torch.maximum(stats[STATS_SUM * n:], step_stats[STATS_SUM * n:], out=stats[STATS_SUM * n:])


class Trainer:
    """Holds parameters, Adam moments, densification statistics and the
    per-view scratch of one rank. ``scene`` provides raw parameters as numpy
    arrays (means3d, features_dc, features_rest [N,15,3], opacity_logits,
    log_scales, rotations)."""

    def __init__(self, scene, device, lrs: LearningRates | None = None, w_l1: float = 1.0,
                 w_ssim: float = 0.2, betas=(0.9, 0.99), eps: float = 1e-8,
                 bias_correction: bool = False, process_group=None, background=(0.0, 0.0, 0.0),
                 comm: str | None = None):
        self.dev = torch.device(device)
        self.n = n = int(scene.means3d.shape[0])
        if scene.features_rest.shape[1:] != (15, 3):
            raise ValueError("the training step stores SH degree 3 (15 rest coefficients)")
        self.sh_degree = int(scene.sh_degree)
        self.lrs = lrs or LearningRates()
        self.w_l1, self.w_ssim = float(w_l1), float(w_ssim)
        # "l1_dssim" (w_l1 L1 + w_ssim D-SSIM) or "mse" (the reference
        # trainer's warm-up loss, scripts/train_scanner_fastgs.py:957-960)
        self.loss_mode = "l1_dssim"
        self.betas, self.eps, self.bias_correction = betas, float(eps), bool(bias_correction)
        self.pg = process_group
        flat = np.concatenate([scene.means3d.reshape(-1), scene.features_dc.reshape(-1),
                               scene.features_rest.reshape(-1), scene.opacity_logits.reshape(-1),
                               scene.log_scales.reshape(-1), scene.rotations.reshape(-1)]).astype(np.float32)
        assert flat.size == FLOATS_PER_GAUSSIAN * n
        d = self.dev
        self.world, self.rank = 1, 0
        if process_group is not None:
            import torch.distributed as dist

            self.world, self.rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        total = FLOATS_PER_GAUSSIAN * n
        # parameters and gradients padded to 16-byte-aligned equal shards: with
        # several ranks the gradients are reduce-scattered, each rank runs Adam
        # on its shard only and the parameters are all-gathered back
        self._per = -(-total // (4 * self.world)) * 4
        padded = self._per * self.world
        self.comm = "local"
        self._symm = None
        if self.world > 1:
            self.comm = comm or os.environ.get("FGS_COMM", "") or default_comm(self.world)
            if self.comm in ("multicast", "p2p", "push", "ce"):
                self._symm = _symmetric_pair(padded, d, process_group, self.comm == "multicast")
                if self._symm is None:
                    self.comm = "nccl"
        if self._symm is not None:
            self.params_pad, self.grads_pad, self._hp, self._hg = self._symm
            self.params_pad.zero_()
            self.grads_pad.zero_()
        else:
            self.params_pad = torch.zeros(padded, device=d)
            self.grads_pad = torch.zeros(padded, device=d)
        self.params_pad[:total].copy_(torch.from_numpy(flat))
        self.params = self.params_pad[:total]
        self.grads = self.grads_pad[:total]
        self._lo, self._hi = shard_range(total, self.world, self.rank)
        # this step's densification statistics of this rank's views: sum
        # |grad_xy|, sum |grad_abs|, visible-view count (3N), max screen radius (N)
        self.step_stats = torch.zeros((STATS_SUM + 1) * n, device=d)
        # running densification statistics of this rank [acc, acc_abs, denom,
        # max_radii] (FastGSDensificationState of scripts/train_scanner_fastgs.py).
        # Sums and maxima commute, so ranks keep their own and global_stats()
        # combines them when densification needs them: no per-step collective.
        self.stats = torch.zeros(4 * n, device=d)
        # Adam moments of this rank's shard
        self.exp_avg = torch.zeros(self._per, device=d)
        self.exp_avg_sq = torch.zeros(self._per, device=d)
        self.opacities = torch.empty(n, device=d)
        self.scales = torch.empty((n, 3), device=d)
        self.quats = torch.empty((n, 4), device=d)
        self.background = torch.tensor(background, dtype=torch.float32, device=d)
        self.step_count = 0
        self.ws = _Grow(d)
        self.k_host = torch.empty(1, dtype=torch.uint64, pin_memory=True)
        self.last_rendered = 0
        self.last_buckets_bound = 0
        # learning-rate group ends, relative to this rank's shard
        ends = np.clip(np.array([3, 6, 51, 52, 55, 59], dtype=np.int64) * n - self._lo, 0,
                       self._hi - self._lo)
        self._group_end = (C.c_int64 * 6)(*ends.tolist())
        # With several ranks and a symmetric-memory exchange, the SH rest
        # coefficients (45 of the 59 floats) are exchanged after the rest of
        # the buffer, while the next render's geometry and binning run on a
        # second stream; that render's colour step waits for them. Everything
        # a caller queues on its own stream after step() sees the whole update.
        # Off by default: at two B200s the geometry kernels slowed by as much
        # as the exchange hid (config 3, views/s: 708.9 without; 644.0 /
        # 700.3 / 709.6 with 1 / 2 / 4 exchange CTAs per SM).
        self.overlap = (self._symm is not None
                        and os.environ.get("FGS_OVERLAP_EXCHANGE", "0") == "1")
        self._geo_stream = torch.cuda.Stream(device=d, priority=-1) if self.overlap else None
        self.rest_blocks_per_sm = int(os.environ.get("FGS_REST_BLOCKS_PER_SM", "4"))
        self._e_front = torch.cuda.Event()  # every rank's non-SH parameters landed
        self._front_pending = False
        self._geo_done = torch.cuda.Event()
        self._set_pieces()
        # instrumentation: CUDA events around chosen launches (same stream),
        # and a count of this library's kernel launches
        self.record = set()
        # forward pass records contributing pairs for the backward pass
        self.contrib_mask = os.environ.get("FGS_CONTRIB_MASK", "1") != "0"
        # bucket samples only where a pixel is still live (fgs_raster_params.sparse_samples)
        self.sparse_samples = os.environ.get("FGS_SPARSE_SAMPLES", "1") != "0"
        self._key_cap = 0  # capacity of the grow-only key buffers
        self.depth_first = os.environ.get("FGS_DEPTH_FIRST", "1") != "0"
        self._k_ready = torch.cuda.Event()  # recorded after each view's key-count copy
        self._scan_done = torch.cuda.Event()
        self._cam_ready = torch.cuda.Event()
        self._g2_ready = torch.cuda.Event()
        self._k_stream = torch.cuda.Stream(device=self.dev)
        self._cam_host = torch.empty(35, dtype=torch.float32, pin_memory=True)
        self._views = 0
        # look-back timeout flags of each view's two sorts (depth order, tile
        # bits), copied back in a two-slot ring: the host reads a view's slot
        # after the next view's key-count wait, which orders after the copies
        self._sort_flags = torch.zeros((2, 2), dtype=torch.int32, pin_memory=True)
        self._flag_views: list[int] = []
        # one view on one rank: Adam fused into the backward pass (no
        # gradient buffer round trip); the gradient buffer is then not written
        self.fuse_adam = os.environ.get("FGS_FUSE_ADAM", "1") != "0"
        self.events: dict[str, list] = {}
        self.launches = 0
        # NVTX ranges around every library call (FGS_NVTX=1), for timeline tools
        self.nvtx = os.environ.get("FGS_NVTX", "0") == "1"

    def full_moments(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Adam moments of every flat element (59 n floats each): this rank's
        shards, all-gathered when the moments are sharded over ranks."""
        self.settle()
        total = FLOATS_PER_GAUSSIAN * self.n
        if self.world == 1:
            return self.exp_avg[:total], self.exp_avg_sq[:total]
        import torch.distributed as dist

        out = []
        for t in (self.exp_avg, self.exp_avg_sq):
            full = torch.empty(self._per * self.world, device=self.dev)
            dist.all_gather_into_tensor(full, t.contiguous(), group=self.pg)
            out.append(full[:total])
        return out[0], out[1]

    def _resize(self, n_new: int, params_new: torch.Tensor, exp_avg_new: torch.Tensor,
                exp_avg_sq_new: torch.Tensor, stats_new: torch.Tensor) -> None:
        """Adopt buffers for n_new Gaussians (densification): the flat
        parameters and the full (unsharded) moments, at least 59 n_new floats
        each, and this rank's running statistics [acc | acc_abs | denom |
        max_radii]; gradients and per-step statistics restart at zero. With
        several ranks every rank calls it with the same parameters and
        moments (the decisions are made on global statistics with one
        generator): each keeps its shard of the moments, and the symmetric
        parameter and gradient buffers are allocated and registered anew."""
        self.settle()
        d = self.dev
        total = FLOATS_PER_GAUSSIAN * n_new
        self.n = n_new
        self._per = -(-total // (4 * self.world)) * 4
        padded = self._per * self.world
        self._symm = None
        if self.comm in ("multicast", "p2p", "push", "ce"):
            self._symm = _symmetric_pair(padded, d, self.pg, self.comm == "multicast")
            if self._symm is None:
                self.comm = "nccl"
        if self._symm is not None:
            self.params_pad, self.grads_pad, self._hp, self._hg = self._symm
        else:
            self.overlap = False
            self.params_pad = torch.empty(padded, device=d)
            self.grads_pad = torch.empty(padded, device=d)
        self.params_pad.zero_()
        self.grads_pad.zero_()
        self.params_pad[:total].copy_(params_new[:total])
        self.params = self.params_pad[:total]
        self.grads = self.grads_pad[:total]
        self._lo, self._hi = shard_range(total, self.world, self.rank)
        self.exp_avg = torch.zeros(self._per, device=d)
        self.exp_avg_sq = torch.zeros(self._per, device=d)
        self.exp_avg[:self._hi - self._lo].copy_(exp_avg_new[self._lo:self._hi])
        self.exp_avg_sq[:self._hi - self._lo].copy_(exp_avg_sq_new[self._lo:self._hi])
        self.stats = stats_new
        self.step_stats = torch.zeros((STATS_SUM + 1) * n_new, device=d)
        self.opacities = torch.empty(n_new, device=d)
        self.scales = torch.empty((n_new, 3), device=d)
        self.quats = torch.empty((n_new, 4), device=d)
        ends = np.clip(np.array([3, 6, 51, 52, 55, 59], dtype=np.int64) * n_new - self._lo, 0,
                       self._hi - self._lo)
        self._group_end = (C.c_int64 * 6)(*ends.tolist())
        self._set_pieces()
        self._vs_zeroed = False

    # kernels each C entry point launches (memsets are not kernels)
    _KERNELS = {"colors": 1, "preprocess": 1, "depth_order": 8, "scan": 3, "duplicate": 1, "tile_prep": 2, "tile_order": 1, "rasterize_forward": 1,
                "loss": 2, "rasterize_backward": 1, "preprocess_backward_train": 1,
                "preprocess_backward_adam": 1, "activate": 1,
                "adam": 1}

    def settle(self) -> None:
        """Close the overlap window of the last step: the next render then
        starts after everything queued on the caller's stream (densification,
        opacity resets, checkpoint loads), not only after the exchange's
        non-SH part."""
        self._front_pending = False

    def _set_pieces(self) -> None:
        """Split this rank's shard [0, per) into the part before the SH rest
        segment, the SH rest segment [6n, 51n) (rounded inwards to 16-byte
        boundaries) and the part after it, each with its own group table."""
        n, lo, per = self.n, self._lo, self._per
        rs = min(max(-(-6 * n // 4) * 4 - lo, 0), per)
        re = max(min(max((51 * n // 4) * 4 - lo, 0), per), rs)
        shard_ends = np.clip(np.array([3, 6, 51, 52, 55, 59], dtype=np.int64) * n - lo, 0,
                             self._hi - lo)
        self._pieces = []
        for off, ln in ((0, rs), (rs, re - rs), (re, per - re)):
            ends = np.clip(shard_ends - off, 0, ln)
            self._pieces.append((off, ln, (C.c_int64 * 6)(*ends.tolist())))
        if self.comm == "ce":
            self._ce_setup(shard_ends)

    def _ce_setup(self, shard_ends) -> None:
        """Copy-engine exchange state: views of every rank's symmetric
        buffers, a staging buffer for the other ranks' gradient shards, the
        pull and push streams, and the shard's chunks (each with its group
        table) that the pipeline moves one by one."""
        world, per, d = self.world, self._per, self.dev
        padded = per * world
        self._peer_g = [self._hg.get_buffer(r, (padded,), torch.float32) for r in range(world)]
        self._peer_p = [self._hp.get_buffer(r, (padded,), torch.float32) for r in range(world)]
        self._stage = torch.empty((max(world - 1, 1), per), device=d)
        if not hasattr(self, "_pull"):
            self._pull = torch.cuda.Stream(device=d)
            self._push = torch.cuda.Stream(device=d)
            self._ce_start, self._ce_done = torch.cuda.Event(), torch.cuda.Event()
        chunks = max(1, int(os.environ.get("FGS_CE_CHUNKS", "4")))
        step = -(-per // (4 * chunks)) * 4
        self._ce_chunks = []
        for off in range(0, per, step):
            ln = min(step, per - off)
            ends = np.clip(shard_ends - off, 0, ln)
            self._ce_chunks.append((off, ln, (C.c_int64 * 6)(*ends.tolist()),
                                    torch.cuda.Event(), torch.cuda.Event()))

    def _ce_exchange(self, lrs, b1, b2) -> None:
        """Reduce-scatter + Adam + all-gather over the copy engines, chunk by
        chunk: the pull stream copies the other ranks' gradients of a chunk of
        this rank's shard into the staging buffer, this stream runs Adam on it
        (gradients summed in rank order), the push stream copies the chunk's
        new parameters into every other rank's buffer; the three overlap
        across chunks."""
        world, rank, lo = self.world, self.rank, self._lo
        main = torch.cuda.current_stream(self.dev)
        others = [r for r in range(world) if r != rank]
        self._ce_start.record(main)
        self._pull.wait_event(self._ce_start)
        self._push.wait_event(self._ce_start)
        for off, ln, ends, ev_in, ev_adam in self._ce_chunks:
            a, b = lo + off, lo + off + ln
            with torch.cuda.stream(self._pull):
                for k, r in enumerate(others):
                    self._stage[k, off:off + ln].copy_(self._peer_g[r][a:b], non_blocking=True)
                ev_in.record(self._pull)
            main.wait_event(ev_in)
            gp = []
            for r in range(world):
                gp.append(_p(self.grads_pad[a:]) if r == rank else _p(self._stage[others.index(r), off:]))
            gpa = (C.c_void_p * world)(*[g.value for g in gp])
            self._call("adam", lib().fgs_adam_step_gathered, ln, world, gpa, _p(self.params_pad[a:]),
                       _p(self.exp_avg[off:]), _p(self.exp_avg_sq[off:]), 6, ends, lrs, b1, b2,
                       self.eps, self.step_count, int(self.bias_correction), self._stream())
            ev_adam.record(main)
            with torch.cuda.stream(self._push):
                self._push.wait_event(ev_adam)
                for r in others:
                    self._peer_p[r][a:b].copy_(self.params_pad[a:b], non_blocking=True)
        self._ce_done.record(self._push)
        main.wait_event(self._ce_done)

    def _exchange(self, off, length, group_end, lrs, b1, b2):
        """Fused exchange + Adam of shard elements [off, off + length)."""
        if length <= 0:
            return
        o4 = (self._lo + off) * 4
        if self.comm == "multicast":
            self._call("adam", lib().fgs_adam_step_multicast, length,
                       _p(self.params_pad[self._lo + off:]),
                       C.c_void_p(self._hp.multicast_ptr + o4),
                       C.c_void_p(self._hg.multicast_ptr + o4), _p(self.exp_avg[off:]),
                       _p(self.exp_avg_sq[off:]), 6, group_end, lrs, b1, b2, self.eps,
                       self.step_count, int(self.bias_correction), self._stream())
        else:
            world = self.world
            pp = (C.c_void_p * world)(*[self._hp.buffer_ptrs[r] + o4 for r in range(world)])
            gp = (C.c_void_p * world)(*[self._hg.buffer_ptrs[r] + o4 for r in range(world)])
            self._call("adam", lib().fgs_adam_step_peers, length, world, self.rank, pp, gp,
                       _p(self.exp_avg[off:]), _p(self.exp_avg_sq[off:]), 6, group_end, lrs, b1,
                       b2, self.eps, self.step_count, int(self.bias_correction), self._stream())

    def _call(self, name, fn, *args):
        ev = None
        if name in self.record:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        check(fn(*args), name)
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        if ev is not None:
            ev[1].record()
            self.events.setdefault(name, []).append(ev)
        self.launches += self._KERNELS.get(name, 0)

    def _begin(self, name):
        if name not in self.record:
            return None
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        return ev

    def _end(self, name, ev):
        if ev is not None:
            ev[1].record()
            self.events.setdefault(name, []).append(ev)

    def kernel_ms(self, name):
        """Mean duration (ms) of the recorded launches of ``name``; clears them."""
        evs = self.events.pop(name, [])
        if not evs:
            return None
        return float(np.mean([a.elapsed_time(b) for a, b in evs]))

    # -- parameter views --------------------------------------------------
    def view(self, name):
        n = self.n
        o = {"means3d": (0, 3 * n, (n, 3)), "features_dc": (3 * n, 6 * n, (n, 3)),
             "features_rest": (6 * n, 51 * n, (n, 15, 3)), "opacity_logits": (51 * n, 52 * n, (n,)),
             "log_scales": (52 * n, 55 * n, (n, 3)), "rotations": (55 * n, 59 * n, (n, 4))}[name]
        return self.params[o[0]:o[1]].view(o[2])

    def grad_view(self, name):
        n = self.n
        o = {"means3d": (0, 3 * n, (n, 3)), "features_dc": (3 * n, 6 * n, (n, 3)),
             "features_rest": (6 * n, 51 * n, (n, 15, 3)), "opacity_logits": (51 * n, 52 * n, (n,)),
             "log_scales": (52 * n, 55 * n, (n, 3)), "rotations": (55 * n, 59 * n, (n, 4))}[name]
        return self.grads[o[0]:o[1]].view(o[2])

    # -- one view ---------------------------------------------------------
    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    def render_view(self, cam, target=None, accumulate=False, loss_out=None, loss_scale=1.0,
                    fused_adam=False, stats=None, metric_map=None, metric_count=None,
                    sort_only=False):
        """Forward (and, with a target, loss + backward accumulated into the
        flat gradient buffer) of one view. Returns the image [3, H*W]. With
        fused_adam the backward pass applies the Adam step (of step number
        self.step_count) to the parameters directly instead of writing the
        gradient buffer: for a step whose gradient is this one view's.
        sort_only stops after the binning sort (self.last_sorted holds the
        sorted keys and values) and returns None."""
        L = lib()
        n, d, ws = self.n, self.dev, self.ws
        W, H = int(cam.width), int(cam.height)
        P = W * H
        gx, gy = tile_grid(W, H)
        T = gx * gy
        main = torch.cuda.current_stream(d)
        # geometry and binning on the second stream while the previous step's
        # SH exchange finishes on this one (multi-rank overlap); else here
        split = self.overlap
        geo = main
        if split and self._front_pending:
            geo = self._geo_stream
            geo.wait_event(self._e_front)
            self._front_pending = False
        st = C.c_void_p(geo.cuda_stream)
        gctx = torch.cuda.stream(geo)
        gctx.__enter__()
        # camera upload on the side stream into one of two device slots: the
        # slot's previous user (two views back) and the pinned staging's last
        # copy are complete, because the host has since waited on a later
        # view's key count, which that stream orders after them
        cm = ws.get("cam%d" % (self._views % 2), 35, torch.float32)
        self._views += 1
        hc = self._cam_host.numpy()
        hc[0:16] = cam.viewmatrix.reshape(-1)
        hc[16:32] = cam.projmatrix.reshape(-1)
        hc[32:35] = cam.campos.reshape(-1)
        cur = geo
        with torch.cuda.stream(self._k_stream):
            cm.copy_(self._cam_host, non_blocking=True)
            self._cam_ready.record(self._k_stream)
        cur.wait_event(self._cam_ready)
        vm, pm, cp = cm[0:16], cm[16:32], cm[32:35]
        self.last_cam = cm  # [view 16 | projection 16 | position 3] of this view
        prm = PreprocessParams(n, self.sh_degree, 15, 1.0, 1.0, float(cam.tan_fovx), float(cam.tan_fovy),
                               W, H, 0, 0)
        vs_in = ws.get("vs_in", 4 * n, torch.float32)
        if not getattr(self, "_vs_zeroed", False) or vs_in.data_ptr() != getattr(self, "_vs_ptr", 0):
            vs_in.zero_()
            self._vs_zeroed, self._vs_ptr = True, vs_in.data_ptr()
        radii = ws.get("radii", n, torch.int32)
        xys = ws.get("xys", 2 * n, torch.float32)
        depths = ws.get("depths", n, torch.float32)
        cov3d = ws.get("cov3d", 6 * n, torch.float32)
        rgb = ws.get("rgb", 3 * n, torch.float32)
        conic = ws.get("conic", 4 * n, torch.float32)
        tiles = ws.get("tiles", n, torch.uint32)
        clamped = ws.get("clamped", 3 * n, torch.uint8)
        vs_out = ws.get("vs_out", 4 * n, torch.float32)
        # activations (sigmoid, exp, normalise) are applied inside the kernels
        if split:
            self._call("preprocess", L.fgs_preprocess_forward_train_geometry, C.byref(prm),
                       _p(self.params), _p(vm), _p(pm), _p(vs_in), _p(radii), _p(xys), _p(depths),
                       _p(cov3d), _p(conic), _p(tiles), _p(vs_out), st)
        else:
            self._call("preprocess", L.fgs_preprocess_forward_train, C.byref(prm), _p(self.params),
                       _p(vm), _p(pm), _p(cp), _p(vs_in), _p(radii), _p(xys), _p(depths),
                       _p(cov3d), _p(rgb), _p(conic), _p(tiles), _p(clamped), _p(vs_out), st)
        cap = self._key_cap
        kb = sort_key_bits(T)
        # depth-first binning: order the Gaussians by depth, emit keys in that
        # order, then sort only the tile bits of the K keys (same result as
        # sorting all bits of keys emitted in index order)
        sort_lo = 32 if self.depth_first else 0

        def key_buffers(c):
            # keys, values, sorted keys and values, sort workspace for c keys
            # (the workspace for c keys serves any count up to c)
            sws_n = int(L.fgs_sort_workspace_bytes(c, kb - sort_lo))
            bufs = (ws.get("keys", c, torch.uint64), ws.get("vals", c, torch.uint32),
                    ws.get("skeys", c, torch.uint64), ws.get("svals", c, torch.uint32),
                    ws.get("sort_ws", sws_n, torch.uint8))
            return [_p(t) for t in bufs], sws_n, bufs

        if cap > 0:
            kp, sws_n, kbufs = key_buffers(cap)  # prepared before the scan: nothing waits on it
        offsets = ws.get("offsets", n, torch.uint32)
        total = ws.get("total", 1, torch.uint64)
        scan_scr = ws.get("scan_scr", int(L.fgs_scan_scratch_bytes(n)), torch.uint8)
        order = None
        scan_in = tiles
        if self.depth_first:
            order = ws.get("depth_order", n, torch.uint32)
            scan_in = ws.get("tiles_in_order", n, torch.uint32)
            dws_n = int(L.fgs_depth_order_workspace_bytes(n))
            dws = ws.get("depth_order_ws", dws_n, torch.uint8)
            self._call("depth_order", L.fgs_depth_order, n, _p(depths), _p(tiles), _p(order), _p(scan_in),
                       _p(dws), dws_n, st)
        self._call("scan", L.fgs_inclusive_scan_u32, n, _p(scan_in), _p(offsets), _p(total), _p(scan_scr), st)
        # the 8-byte count goes to the host on a side stream, so that the copy
        # does not sit between the scan and the next launch on this stream
        self._scan_done.record(cur)
        with torch.cuda.stream(self._k_stream):
            self._k_stream.wait_event(self._scan_done)
            self.k_host.copy_(total, non_blocking=True)
            self._k_ready.record(self._k_stream)
        k_ready = self._k_ready
        # Duplicate-with-keys runs before the host knows K, into grow-only
        # buffers of the capacity the previous views needed (its writes stop at
        # the capacity); the host only waits for the count, and repeats the
        # launch with larger buffers in the rare view that outgrows them.
        def dup(c, kp):
            if order is None:
                self._call("duplicate", L.fgs_duplicate_with_keys, n, 1.0, gx, gy, _p(xys), _p(depths),
                           _p(offsets), _p(conic), _p(tiles), c, kp[0], kp[1], st)
            else:
                self._call("duplicate", L.fgs_duplicate_with_keys_ordered, n, 1.0, gx, gy, _p(xys),
                           _p(depths), _p(order), _p(offsets), _p(conic), _p(tiles), c, kp[0], kp[1], st)

        if cap > 0:
            dup(cap, kp)
        k_ready.synchronize()  # the one host sync: K sizes the sort and the bucket arrays
        self._check_sort_flags()  # every earlier view's flag copies have landed
        K = int(self.k_host.item())
        self.last_rendered = K
        if K > cap:
            cap = self._key_cap = K + K // 4 + 1024
            kp, sws_n, kbufs = key_buffers(cap)
            dup(cap, kp)
        slot = self._sort_flags[(self._views - 1) % 2]
        slot.zero_()
        if self.depth_first:
            slot[0:1].copy_(dws[:4].view(torch.int32), non_blocking=True)
        if K > 0:
            self._call("sort", L.fgs_sort_pairs_bits, K, sort_lo, kb, *kp, sws_n, st)
            slot[1:2].copy_(kbufs[4][:4].view(torch.int32), non_blocking=True)
        self._flag_views.append(self._views - 1)
        gctx.__exit__(None, None, None)
        if geo is not main:
            self._geo_done.record(geo)
            main.wait_event(self._geo_done)
        cur, st = main, C.c_void_p(main.cuda_stream)
        if split:
            # colours from the SH coefficients, which the previous step's
            # exchange has finished writing on this stream
            self._call("colors", L.fgs_preprocess_colors_train, C.byref(prm), _p(self.params),
                       _p(cp), _p(tiles), _p(rgb), _p(clamped), st)
        if target is not None:
            # the raster-gradient accumulators are zeroed on the side stream
            # while this stream sorts and renders (every earlier use of them
            # finished before this view's scan, which the host just saw)
            o1 = -(-2 * n // 4) * 4
            o2 = o1 + -(-3 * n // 4) * 4
            g2 = ws.get("g_raster", o2 + 8 * n, torch.float32)
            with torch.cuda.stream(self._k_stream):
                g2.zero_()
                self._g2_ready.record(self._k_stream)
        img = ws.get("img", 3 * P, torch.float32)
        if K == 0:
            img.view(3, P).copy_(self.background.view(3, 1).expand(3, P))
            return img
        skeys, svals = kbufs[2][:K], kbufs[3][:K]
        self.last_sorted = (skeys, svals)
        self.launches += 2 + (kb - sort_lo + 7) // 8  # histogram, digit scan, one pass per digit
        if sort_only:
            return None
        ranges = ws.get("ranges", 2 * T, torch.uint32)
        bcount = ws.get("bcount", T, torch.uint32)
        boffs = ws.get("boffs", T, torch.uint32)
        bsum = ws.get("bsum", 1, torch.uint64)
        # every tile has at most ceil(n_t/32) <= n_t/32 + 1 buckets: size the
        # bucket arrays by that bound instead of reading the sum back; entries
        # past the real sum get an invalid tile id (the backward pass skips them)
        Bmax = (K + 31) // 32 + T
        self.last_buckets_bound = Bmax
        b2t = ws.get("b2t", Bmax, torch.uint32)
        order = ws.get("tile_order", T, torch.uint32)
        self._call("tile_prep", L.fgs_tile_prep_ordered, K, T, _p(skeys), _p(ranges), _p(bcount),
                   _p(boffs), _p(bsum), _p(order), _p(b2t), Bmax, st)
        samp_t = ws.get("samp_t", Bmax * 256, torch.float32)
        samp_ar = ws.get("samp_ar", Bmax * 768, torch.float32)
        final_t = ws.get("final_t", P, torch.float32)
        ncontrib = ws.get("ncontrib", P, torch.uint32)
        maxc = ws.get("maxc", T, torch.uint32)
        pixc = ws.get("pixc", 3 * P, torch.float32)
        cm_ptr = None
        if self.contrib_mask:
            cm_ptr = ws.get("contrib_mask", Bmax * 256, torch.uint32).data_ptr()
        # FastGS metric counting (a second render of a sampled view,
        # scripts/train_scanner_fastgs.py:313): metric_map [P] int32 in,
        # metric_count [n] int32 out
        get_flag = int(metric_map is not None)
        # sparse samples: pixels that terminated before a bucket get no sample
        # writes there, and the backward pass reads none
        rp = RasterParams(W, H, T, Bmax, n, get_flag, order.data_ptr(), cm_ptr, int(self.sparse_samples))
        self._call("rasterize_forward", L.fgs_rasterize_forward, C.byref(rp), _p(ranges), _p(svals), _p(boffs), _p(xys), _p(rgb), _p(conic),
            _p(self.background), _p(metric_map), _p(b2t), _p(samp_t), _p(samp_ar), _p(final_t), _p(ncontrib),
            _p(maxc), _p(pixc), _p(img), _p(metric_count), st)
        if target is None:
            return img
        # loss and its gradient w.r.t. the image
        dimg = ws.get("dimg", 3 * P, torch.float32)
        lscr = ws.get("loss_scr", int(L.fgs_loss_scratch_bytes(W, H)) // 4 + 1, torch.float32)
        lout = loss_out if loss_out is not None else ws.get("loss_out", 4, torch.float32)
        if self.loss_mode == "mse":
            self._call("loss", L.fgs_mse_loss, W, H, _p(img), _p(target), loss_scale, _p(lout),
                       _p(dimg), _p(lscr), st)
        else:
            self._call("loss", L.fgs_l1_dssim_loss, W, H, _p(img), _p(target), self.w_l1 * loss_scale,
                       self.w_ssim * loss_scale, _p(lout), _p(dimg), _p(lscr), st)
        # backward
        # one zeroed buffer, each part starting on a 16-byte boundary (the
        # kernels read the conic and viewspace gradients as float4)
        cur.wait_event(self._g2_ready)
        dmeans2d, dcolors = g2[:2 * n], g2[o1:o1 + 3 * n]
        dconic, dvs = g2[o2:o2 + 4 * n], g2[o2 + 4 * n:o2 + 8 * n]
        self.raster_grads = (dmeans2d, dcolors, dconic, dvs)
        self._call("rasterize_backward", L.fgs_rasterize_backward, C.byref(rp), _p(ranges), _p(svals), _p(boffs), _p(xys), _p(rgb), _p(conic),
            _p(self.background), _p(dimg), _p(b2t), _p(samp_t), _p(samp_ar), _p(final_t),
            _p(ncontrib), _p(maxc), _p(pixc), _p(dmeans2d), _p(dcolors), _p(dconic), _p(dvs), st)
        if fused_adam:
            lr = self.lrs
            lrs = (C.c_float * 6)(lr.means, lr.dc, lr.rest, lr.opacity, lr.scales, lr.rotations)
            self._call("preprocess_backward_adam", L.fgs_preprocess_backward_adam, C.byref(prm),
                       _p(vm), _p(pm), _p(cp),
                       _p(cov3d), _p(dcolors), _p(dmeans2d), _p(dconic), _p(dvs), _p(radii),
                       _p(clamped), _p(self.params), _p(self.exp_avg), _p(self.exp_avg_sq), lrs,
                       float(self.betas[0]), float(self.betas[1]), self.eps, self.step_count,
                       int(self.bias_correction), _p(self.step_stats if stats is None else stats), st)
            return img
        if self.comm == "push":
            # the gradients go straight into their owners' buffers
            gp = (C.c_void_p * self.world)(*self._hg.buffer_ptrs)
            self._call("preprocess_backward_train", L.fgs_preprocess_backward_push, C.byref(prm),
                       _p(self.params), _p(vm), _p(pm), _p(cp), _p(cov3d), _p(dcolors),
                       _p(dmeans2d), _p(dconic), _p(dvs), _p(radii), _p(clamped), self.world,
                       self._per, gp, _p(self.step_stats), st)
            return img
        self._call("preprocess_backward_train", L.fgs_preprocess_backward_train, C.byref(prm),
                   _p(self.params), _p(vm), _p(pm), _p(cp), _p(cov3d), _p(dcolors), _p(dmeans2d),
                   _p(dconic), _p(dvs), _p(radii), _p(clamped), int(bool(accumulate)),
                   _p(self.grads), _p(self.step_stats), st)
        return img

    def _check_sort_flags(self) -> None:
        """Raise if a sort of an earlier view reported a look-back timeout
        (the flag fgs_sort_status reads). Call only where the copies of those
        flags are known to have landed."""
        views, self._flag_views = self._flag_views, []
        for v in views:
            f = self._sort_flags[v % 2]
            if int(f[0]) or int(f[1]):
                raise RuntimeError(f"sort of view {v} failed (status {_lib.FGS_ERR_TIMEOUT}): a "
                                   "look-back wait gave up after its poll limit")

    # -- checkpoint ---------------------------------------------------------
    def state_dict(self) -> dict:
        """Everything a resumed run needs, as CPU tensors: the raw parameters
        [59 n], the full Adam moments (all-gathered when sharded), the running
        densification statistics over every rank's views, the step count.
        A collective with several ranks (every rank calls it; all get the
        same dictionary)."""
        m, v = self.full_moments()
        return {"n": self.n, "step_count": self.step_count, "sh_degree": self.sh_degree,
                "params": self.params.detach().cpu().clone(), "exp_avg": m.cpu().clone(),
                "exp_avg_sq": v.cpu().clone(), "stats": self.global_stats().cpu(),
                "betas": tuple(self.betas), "eps": self.eps,
                "bias_correction": self.bias_correction}

    def load_state_dict(self, state: dict) -> None:
        """Resume from state_dict() (of this or another world size): every
        rank adopts the parameters and its shard of the moments; the
        statistics go to rank 0 (the others start at zero, so their sum and
        maximum over ranks are the saved ones)."""
        self.settle()
        d = self.dev
        n = int(state["n"])
        total = FLOATS_PER_GAUSSIAN * n
        params = state["params"].to(d, torch.float32).reshape(-1)[:total]
        m = state["exp_avg"].to(d, torch.float32).reshape(-1)[:total]
        v = state["exp_avg_sq"].to(d, torch.float32).reshape(-1)[:total]
        stats = state["stats"].to(d, torch.float32).reshape(-1).clone()
        if self.rank != 0:
            stats.zero_()
        self._resize(n, params, m, v, stats)
        self.step_count = int(state["step_count"])
        self.sh_degree = int(state.get("sh_degree", self.sh_degree))

    def check_sort_status(self) -> None:
        """Synchronise and raise if any sort since the last check timed out."""
        torch.cuda.current_stream(self.dev).synchronize()
        self._check_sort_flags()

    def global_stats(self) -> torch.Tensor:
        """Densification statistics over every rank's views (sum; max for the
        screen radius), as a new tensor [acc, acc_abs, denom, max_radii]."""
        out = self.stats.clone()
        if self.world > 1:
            allreduce_stats(out, self.n, self.pg)
        return out

    # -- full step --------------------------------------------------------
    def activate(self):
        """Activated copies of the parameters (self.opacities, self.scales,
        self.quats) for callers that want them; the step's own kernels apply
        the activations to the raw parameters themselves."""
        self.settle()
        self._call("activate", lib().fgs_activate_params, self.n, _p(self.params), _p(self.opacities),
                   _p(self.scales), _p(self.quats), self._stream())

    def step(self, cams, targets, loss_out=None):
        """One optimisation step over ``cams`` (the whole batch; this rank
        renders its share). ``targets[i]`` is the [3, H*W] float32 target of
        cams[i] on this device (None for views of other ranks). The loss of
        the local views (sum) lands in loss_out[0] (device)."""
        world, rank = self.world, self.rank
        mine = local_views(len(cams), world, rank)
        scale = 1.0 / max(len(cams), 1)  # mean loss over the whole batch
        if self.fuse_adam and world == 1 and len(mine) == 1:
            # the gradient is this one view's: Adam runs inside its backward
            # pass, and the view's densification statistics go straight into
            # the running ones (the same sums and maxima as folding them)
            self.step_count += 1
            self.render_view(cams[mine[0]], targets[mine[0]], loss_out=loss_out, loss_scale=scale,
                             fused_adam=True, stats=self.stats)
            return 1
        self.step_stats.zero_()
        if not mine and self.comm != "push":
            self.grads.zero_()
        for j, v in enumerate(mine):
            lo = None
            if loss_out is not None:
                lo = loss_out if j == 0 else self.ws.get("loss_tmp", 4, torch.float32)
            self.render_view(cams[v], targets[v], accumulate=j > 0, loss_out=lo, loss_scale=scale)
            if loss_out is not None and j > 0:
                loss_out[:3].add_(lo[:3])
        lo, hi = self._lo, self._hi
        fold_stats(self.stats, self.step_stats, self.n)
        self.step_count += 1
        lr = self.lrs
        lrs = (C.c_float * 6)(lr.means, lr.dc, lr.rest, lr.opacity, lr.scales, lr.rotations)
        b1, b2 = float(self.betas[0]), float(self.betas[1])
        if self.comm == "ce":
            ev = self._begin("exchange")
            self._hp.barrier(channel=0)
            self._ce_exchange(lrs, b1, b2)
            self._hp.barrier(channel=1)
            self._end("exchange", ev)
            return len(mine)
        if self.comm == "push":
            # every rank's gradients pushed -> the owner's Adam on its summed
            # shard, which clears it and stores the parameters to every rank
            ev = self._begin("exchange")
            self._hp.barrier(channel=0)
            world, lo = self.world, self._lo
            pp = (C.c_void_p * world)(*[self._hp.buffer_ptrs[r] + 4 * lo for r in range(world)])
            mc = getattr(self._hp, "multicast_ptr", 0) if world > 2 else 0
            self._call("adam", lib().fgs_adam_step_owner, self._per, world, self.rank, pp,
                       C.c_void_p(mc + 4 * lo) if mc else None, _p(self.grads_pad[lo:]),
                       _p(self.exp_avg), _p(self.exp_avg_sq), 6, self._group_end, lrs, b1, b2,
                       self.eps, self.step_count, int(self.bias_correction), self._stream())
            self._hp.barrier(channel=1)
            self._end("exchange", ev)
            return len(mine)
        if self.comm in ("multicast", "p2p"):
            # every rank's gradients written -> fused exchange + Adam -> every
            # rank's parameter broadcast landed (also guards the next step's
            # gradient writes against peers still reading these)
            ev = self._begin("exchange")
            self._hp.barrier(channel=0)
            if self.overlap:
                # the non-SH parts first; the next render's geometry starts
                # once every rank has them, while the SH rest part moves
                front, rest, back = self._pieces
                self._exchange(front[0], front[1], front[2], lrs, b1, b2)
                self._exchange(back[0], back[1], back[2], lrs, b1, b2)
                self._hp.barrier(channel=1)
                self._e_front.record(torch.cuda.current_stream(self.dev))
                self._front_pending = True
                # a small grid, so that the next render's geometry kernels
                # find free SMs while this one strides over the SH shard
                check(lib().fgs_set_exchange_grid(self.rest_blocks_per_sm), "set_exchange_grid")
                self._exchange(rest[0], rest[1], rest[2], lrs, b1, b2)
                check(lib().fgs_set_exchange_grid(0), "set_exchange_grid")
                self._hp.barrier(channel=2)
            elif lr.rest < 0.0:
                # the SH rest group does not step (the reference's cadence,
                # scripts/train_scanner_fastgs.py:166-171, steps it every 16th
                # iteration at most): its gradients are dropped, as there, so
                # only the other parts of the shard cross NVLink
                front, _, back = self._pieces
                self._exchange(front[0], front[1], front[2], lrs, b1, b2)
                self._exchange(back[0], back[1], back[2], lrs, b1, b2)
                self._hp.barrier(channel=1)
            else:
                self._exchange(0, self._per, self._group_end, lrs, b1, b2)
                self._hp.barrier(channel=1)
            self._end("exchange", ev)
            return len(mine)
        if world > 1:
            ev = self._begin("reduce")
            reduce_scatter_grads(self.grads_pad, world, rank, self.pg)
            self._end("reduce", ev)
        self._call("adam", lib().fgs_adam_step, hi - lo, _p(self.params_pad[lo:]),
                   _p(self.grads_pad[lo:]), _p(self.exp_avg), _p(self.exp_avg_sq), 6,
                   self._group_end, lrs, b1, b2, self.eps, self.step_count,
                   int(self.bias_correction), self._stream())
        if world > 1:
            ev = self._begin("allgather")
            allgather_params(self.params_pad, world, rank, self.pg)
            self._end("allgather", ev)
        return len(mine)
