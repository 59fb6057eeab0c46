"""FastGS densification of a Trainer's Gaussians on the device.

The reference runs it on the host over NumPy copies of every tensor
(scripts/train_scanner_fastgs.py:470-795, FastGSDensificationState and
ScannerFastGSOptimizerPolicy); here the parameters, Adam moments and running
statistics stay on the GPU: the decision masks are one kernel
(fgs_densify_masks / fgs_prune_masks), pruning, cloning and splitting are row
gathers over the flat layouts (fgs_gather_rows), the split children are one
kernel (fgs_split_fixup) and the opacity cap another (fgs_opacity_cap). The
host keeps the pieces that consume the caller's random generator, in the
reference's order and with the same arguments: rng.normal for the split
offsets (scaled by the sources' scales) and rng.choice for the weighted prune
budget, so a run with the same generator makes the same choices.

Two index mismatches of the reference are resolved as the original 3DGS
does: rows cloned in a call are appended after the split candidates and are
never split (the split masks are padded with False), and the pruning scores
follow their rows through the clone, split and prune steps (appended rows
score 0).

Functions take the Trainer (fastgs_core_b200.train.Trainer) and numpy
arrays for host-side scores; they return the reference's statistics dicts.
Under view-sharded data parallelism every rank calls them in the same order
with an equally seeded generator: decisions use the all-reduced statistics
and rank 0's scores, parameters are replicated, and the Adam moments are
all-gathered for the row gathers and re-sharded by Trainer._resize.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import check, lib

PARAM_WIDTHS = (3, 3, 45, 1, 3, 4)  # means, dc, sh rest, opacity logit, log-scale, rotation
STATS_WIDTHS = (1, 1, 1, 1)          # acc, acc_abs, denom, max_radii


@dataclass
class DensifyArgs:
    """The arguments densify_and_prune_fastgs reads (scripts/train_scanner_fastgs.py:827-849
    defaults)."""
    grad_thresh: float = 2.0e-4
    grad_abs_thresh: float = 1.2e-3
    dense: float = 0.01
    importance_score_threshold: float = 5.0
    split_factor: int = 2
    min_opacity: float = 0.005
    max_screen_size: float = 20.0
    max_world_scale_factor: float = 0.1
    prune_budget_factor: float = 0.5
    opacity_cap_after_densify: float = 0.82


def _p(t):
    return C.c_void_p(t.data_ptr())


def _gather(src: torch.Tensor, n_in: int, n_out: int, index: torch.Tensor, widths, size: int) -> torch.Tensor:
    dst = torch.zeros(size, dtype=torch.float32, device=src.device)
    w = (C.c_int32 * len(widths))(*widths)
    check(lib().fgs_gather_rows(n_in, n_out, _p(index), len(widths), w, _p(src), _p(dst),
                                torch.cuda.current_stream(src.device).cuda_stream), "gather_rows")
    return dst


def _padded(n: int) -> int:
    return -(-59 * n // 4) * 4


def _apply_rows(tr, param_index: np.ndarray, moment_index: np.ndarray, keep_stats: bool) -> None:
    """Rebuild the trainer's buffers with row j = old row param_index[j]
    (moments: moment_index[j], -1 = zeros); statistics follow the rows when
    keep_stats, else restart at zero (reset_densification_buffers)."""
    n_in, n_out = tr.n, int(param_index.size)
    dev = tr.dev
    pi = torch.from_numpy(param_index.astype(np.int64)).to(dev)
    mi = torch.from_numpy(moment_index.astype(np.int64)).to(dev)
    size = _padded(n_out)
    params = _gather(tr.params_pad, n_in, n_out, pi, PARAM_WIDTHS, size)
    m_full, v_full = tr.full_moments()  # all-gathered when sharded over ranks
    m = _gather(m_full, n_in, n_out, mi, PARAM_WIDTHS, size)
    v = _gather(v_full, n_in, n_out, mi, PARAM_WIDTHS, size)
    if keep_stats:
        stats = _gather(tr.stats, n_in, n_out, pi, STATS_WIDTHS, 4 * n_out)
    else:
        stats = torch.zeros(4 * n_out, device=dev)
    tr._resize(n_out, params, m, v, stats)


def prune_points(tr, prune_mask: np.ndarray, score: np.ndarray | None = None):
    """prune_points (scripts/train_scanner_fastgs.py:510-537). Returns the
    pruned score array (or None)."""
    tr.settle()
    prune_mask = np.asarray(prune_mask, bool)
    if prune_mask.size == 0 or not np.any(prune_mask):
        return score
    keep = np.flatnonzero(~prune_mask)
    _apply_rows(tr, keep, keep, keep_stats=True)
    return None if score is None else score[keep]


def _append_copies(tr, sources: np.ndarray, score):
    """append_new_points with copies of rows `sources` (:477-507): moments of
    the new rows start at zero, the statistics restart at zero."""
    n = tr.n
    base = np.arange(n, dtype=np.int64)
    _apply_rows(tr, np.concatenate([base, sources]),
                np.concatenate([base, np.full(sources.size, -1, np.int64)]), keep_stats=False)
    if score is not None:
        score = np.concatenate([score, np.zeros(sources.size, np.float32)])
    return score


def densify_and_clone(tr, metric_mask, clone_filter, score=None):
    """densify_and_clone_fastgs (:540-566)."""
    tr.settle()
    selected = np.asarray(metric_mask, bool) & np.asarray(clone_filter, bool)
    if not np.any(selected):
        return 0, score
    score = _append_copies(tr, np.flatnonzero(selected), score)
    return int(selected.sum()), score


def densify_and_split(tr, metric_mask, split_filter, rng, split_factor: int, score=None):
    """densify_and_split_fastgs (:569-618)."""
    tr.settle()
    selected = np.asarray(metric_mask, bool) & np.asarray(split_filter, bool)
    if selected.size < tr.n:
        selected = np.concatenate([selected, np.zeros(tr.n - selected.size, bool)])
    if not np.any(selected):
        return 0, 0, score
    src = np.flatnonzero(selected)
    n0 = tr.n
    # the sources' scales, as the reference's rng.normal(scale=...) consumes them
    ls_seg = tr.params[52 * n0:55 * n0].view(n0, 3)
    log_scales = ls_seg[torch.from_numpy(src).to(tr.dev)].cpu().numpy()
    scales = np.exp(log_scales).astype(np.float32)
    repeated_scales = np.repeat(scales, split_factor, axis=0)
    samples = rng.normal(loc=0.0, scale=repeated_scales).astype(np.float32)
    children = np.repeat(src, split_factor)
    score = _append_copies(tr, children, score)
    m = children.size
    sd = torch.from_numpy(np.ascontiguousarray(samples)).to(tr.dev)
    check(lib().fgs_split_fixup(tr.n, n0, m, _p(sd), int(split_factor), _p(tr.params_pad),
                                torch.cuda.current_stream(tr.dev).cuda_stream), "split_fixup")
    score = prune_points(tr, np.concatenate([selected, np.zeros(m, bool)]), score)
    return int(src.size), int(m), score


def cap_opacity_logits(tr, opacity_cap: float):
    """cap_opacity_logits (:621-638): logit(min(opacity, cap)); the opacity
    moments restart at zero (with sharded moments: this rank's part of the
    opacity segment)."""
    tr.settle()
    sharded = tr.world > 1
    check(lib().fgs_opacity_cap(tr.n, float(opacity_cap), _p(tr.params_pad),
                                None if sharded else _p(tr.exp_avg),
                                None if sharded else _p(tr.exp_avg_sq),
                                torch.cuda.current_stream(tr.dev).cuda_stream), "opacity_cap")
    if sharded:
        a, b = max(51 * tr.n, tr._lo), min(52 * tr.n, tr._hi)
        if a < b:
            tr.exp_avg[a - tr._lo:b - tr._lo].zero_()
            tr.exp_avg_sq[a - tr._lo:b - tr._lo].zero_()


def reset_opacity_logits(tr, reset_value: float):
    """reset_opacity_logits (:640-658): the same operation as the cap."""
    tr.settle()
    cap_opacity_logits(tr, reset_value)


def _masks(tr, fn_name, *args) -> np.ndarray:
    out = torch.empty(tr.n, dtype=torch.uint8, device=tr.dev)
    fn = getattr(lib(), fn_name)
    check(fn(tr.n, *args, _p(out), torch.cuda.current_stream(tr.dev).cuda_stream), fn_name)
    return out.cpu().numpy()


def densify_and_prune_fastgs(tr, args: DensifyArgs, scene_extent: float, importance_score,
                             pruning_score, rng) -> dict:
    """densify_and_prune_fastgs (:661-745) on the running statistics of
    every rank's views (tr.global_stats(); the trainer's own with one rank).
    With several ranks every rank calls it with the same scores and an
    equally seeded generator, so all make the same choices."""
    tr.settle()
    imp = torch.as_tensor(np.asarray(importance_score, np.float32), device=tr.dev)
    gstats = tr.global_stats() if tr.world > 1 else tr.stats
    mk = _masks(tr, "fgs_densify_masks", _p(tr.params_pad), _p(gstats), _p(imp),
                float(args.grad_thresh), float(args.grad_abs_thresh),
                float(args.dense * scene_extent), float(args.importance_score_threshold))
    clone_sel = (mk & 1) != 0
    split_sel = (mk & 2) != 0
    metric = (mk & 4) != 0
    score = None if pruning_score is None else np.asarray(pruning_score, np.float32).copy()
    cloned, score = densify_and_clone(tr, metric, clone_sel, score)
    split_sources, split_children, score = densify_and_split(tr, metric, split_sel, rng,
                                                             int(args.split_factor), score)
    n = tr.n
    gstats = tr.global_stats() if tr.world > 1 else tr.stats
    pm = _masks(tr, "fgs_prune_masks", _p(tr.params_pad), _p(gstats[3 * n:]),
                float(args.min_opacity), float(args.max_screen_size),
                float(args.max_world_scale_factor * scene_extent if args.max_world_scale_factor > 0 else 0.0))
    opacity_prune = (pm & 1) != 0
    screen_prune = (pm & 2) != 0
    world_prune = (pm & 4) != 0
    prune = opacity_prune | screen_prune | world_prune
    to_remove = int(prune.sum())
    budget = int(args.prune_budget_factor * to_remove)
    removed = 0
    if budget > 0 and score is not None and score.size > 0:
        weights = (1.0 / (1.0e-6 + (1.0 - score))).astype(np.float32)
        cand = np.flatnonzero(prune)
        if cand.size > 0:
            w = weights[cand]
            w = w / max(float(np.sum(w)), 1.0e-6)
            chosen = rng.choice(cand, size=min(budget, cand.size), replace=False, p=w)
            final = np.zeros_like(prune)
            final[chosen] = True
            final &= prune
            removed = int(final.sum())
            score = prune_points(tr, final, score)
    cap_opacity_logits(tr, args.opacity_cap_after_densify)
    return {"metric_hits": int(metric.sum()), "clone_candidates": int(clone_sel.sum()),
            "split_candidates": int(split_sel.sum()), "cloned": cloned,
            "split_sources": split_sources, "split_children": split_children,
            "opacity_prune_candidates": int(opacity_prune.sum()),
            "screen_prune_candidates": int(screen_prune.sum()),
            "world_prune_candidates": int(world_prune.sum()),
            "total_prune_candidates": to_remove, "prune_budget": budget,
            "actual_removed": removed}


def compute_gaussian_scores_fastgs(tr, cams, targets, camera_indices, loss_thresh: float,
                                   densify: bool):
    """compute_gaussian_scores_fastgs (:268-340): for each sampled view, the
    render, the min-max normalised per-pixel L1 map thresholded into a metric
    map, a second render counting each Gaussian's metric pixels, and the
    scores folded over the views (importance = floor(counts / views) when
    densify, pruning = min-max normalised sum of photometric loss x counts).
    targets[i] is the [3, H*W] float32 device target of cams[i]. Returns
    (importance or None, pruning) as numpy arrays."""
    tr.settle()
    L = lib()
    n, dev = tr.n, tr.dev
    st = torch.cuda.current_stream(dev).cuda_stream
    counts = torch.zeros(n, device=dev)
    score = torch.zeros(n, device=dev)
    mcount = torch.empty(n, dtype=torch.int32, device=dev)
    idx = [int(i) for i in np.asarray(camera_indices).reshape(-1)]
    if not idx:
        z = np.zeros(n, np.float32)
        return (z if densify else None), z
    for i in idx:
        cam, target = cams[i], targets[i]
        P = cam.width * cam.height
        pred = tr.render_view(cam).clone()
        mmap = torch.empty(P, dtype=torch.int32, device=dev)
        l1 = torch.empty(1, device=dev)
        scratch = torch.empty(P + 2, device=dev)
        check(L.fgs_metric_map(P, _p(pred), _p(target), float(loss_thresh), _p(mmap), _p(l1),
                               _p(scratch), st), "metric_map")
        tr.render_view(cam, metric_map=mmap, metric_count=mcount)
        check(L.fgs_score_accumulate(n, _p(mcount), _p(l1), 3 * P, _p(counts), _p(score), st),
              "score_accumulate")
    imp = torch.empty(n, device=dev)
    pruning = torch.empty(n, device=dev)
    fin = torch.empty(2, dtype=torch.int32, device=dev)
    check(L.fgs_score_finalize(n, _p(counts), _p(score), len(idx), _p(imp) if densify else None,
                               _p(pruning), _p(fin), st), "score_finalize")
    if tr.world > 1:
        # every rank rendered the same views; the float sums may still differ
        # in their last bits between ranks, so all use rank 0's scores
        import torch.distributed as dist

        dist.broadcast(imp, 0, group=tr.pg)
        dist.broadcast(pruning, 0, group=tr.pg)
    return (imp.cpu().numpy() if densify else None), pruning.cpu().numpy()


def final_prune_fastgs(tr, min_opacity: float, pruning_score, score_thresh: float,
                       min_gaussians: int) -> dict:
    """final_prune_fastgs (:748-795)."""
    tr.settle()
    n = tr.n
    logits = tr.params[51 * n:52 * n].cpu().numpy()
    opacities = (1.0 / (1.0 + np.exp(-logits))).astype(np.float32)
    pruning_score = np.asarray(pruning_score, np.float32)
    opacity_mask = opacities < min_opacity
    score_mask = pruning_score > score_thresh
    prune = opacity_mask | score_mask
    total = int(prune.size)
    requested = int(prune.sum())
    if total == 0:
        return {"total": 0, "opacity_hits": 0, "score_hits": 0, "requested_remove": 0,
                "actual_remove": 0, "kept": 0}
    min_keep = min(max(int(min_gaussians), 0), total)
    if total - requested < min_keep:
        keep_priority = opacities - pruning_score
        keep_indices = np.argsort(keep_priority)[::-1][:min_keep]
        actual = np.ones(total, bool)
        actual[keep_indices] = False
    else:
        actual = prune
    removed = int(actual.sum())
    prune_points(tr, actual)
    return {"total": total, "opacity_hits": int(opacity_mask.sum()), "score_hits": int(score_mask.sum()),
            "requested_remove": requested, "actual_remove": removed, "kept": total - removed}
