"""CPU restatement of the reference's FastGS densification (test
infrastructure only: the checker for fastgs_core_b200.densify).

Follows scripts/train_scanner_fastgs.py: prune_points (:510-537),
append_new_points (:477-507), densify_and_clone_fastgs (:540-566),
densify_and_split_fastgs (:569-618), cap_opacity_logits (:621-638),
reset_opacity_logits (:640-658), densify_and_prune_fastgs (:661-745) and
final_prune_fastgs (:748-795), on numpy arrays:

  params: means3d [n,3], features_dc [n,3], features_rest [n,15,3],
          opacity_logits [n], log_scales [n,3], rotations [n,4]
  adam:   {name: (m, v)} with the same shapes
  stats:  max_radii2d [n], xyz_grad_accum [n], xyz_grad_accum_abs [n],
          denom [n], tmp_radii [n] or None

Two reference index mismatches are resolved as the original 3DGS does, and
the GPU path does the same:
  * densify_and_split_fastgs selects with masks of the pre-clone length; the
    rows cloned in the same call are appended after them and are never split
    (the masks are padded with False);
  * the prune budget's weights index the pre-densification pruning scores
    with post-densification row ids; scores follow their rows through the
    clone, split and prune steps, and appended rows score 0.
The random draws (rng.normal for split offsets, rng.choice for the prune
budget) are made in the reference's order with the caller's generator.
"""
from __future__ import annotations

import numpy as np

PARAMS = ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations")


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def logit(p):
    """scripts/train_scanner_fixed.py:157-159."""
    p = np.clip(p, 1.0e-6, 1.0 - 1.0e-6)
    return np.log(p / (1.0 - p))


def quat_to_rotmat(quat):
    """scripts/train_scanner_fastgs.py:189-201."""
    q = quat / np.maximum(np.linalg.norm(quat, axis=1, keepdims=True), 1.0e-8)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    rot = np.empty((q.shape[0], 3, 3), dtype=np.float32)
    rot[:, 0, 0] = 1.0 - 2.0 * (y * y + z * z)
    rot[:, 0, 1] = 2.0 * (x * y - z * w)
    rot[:, 0, 2] = 2.0 * (x * z + y * w)
    rot[:, 1, 0] = 2.0 * (x * y + z * w)
    rot[:, 1, 1] = 1.0 - 2.0 * (x * x + z * z)
    rot[:, 1, 2] = 2.0 * (y * z - x * w)
    rot[:, 2, 0] = 2.0 * (x * z - y * w)
    rot[:, 2, 1] = 2.0 * (y * z + x * w)
    rot[:, 2, 2] = 1.0 - 2.0 * (x * x + y * y)
    return rot


class State:
    def __init__(self, params, adam, stats, score=None):
        self.params = {k: np.asarray(v, np.float32).copy() for k, v in params.items()}
        self.adam = {k: (np.asarray(m, np.float32).copy(), np.asarray(v, np.float32).copy())
                     for k, (m, v) in adam.items()}
        self.stats = {k: (None if v is None else np.asarray(v, np.float32).copy())
                      for k, v in stats.items()}
        self.score = None if score is None else np.asarray(score, np.float32).copy()

    @property
    def n(self):
        return self.params["means3d"].shape[0]

    def reset_stats(self):
        """reset_densification_buffers (:470-474)."""
        n = self.n
        for k in ("max_radii2d", "xyz_grad_accum", "xyz_grad_accum_abs", "denom"):
            self.stats[k] = np.zeros(n, np.float32)


def prune_points(st: State, prune_mask):
    if prune_mask.size == 0 or not np.any(prune_mask):
        return
    keep = ~prune_mask
    for k in PARAMS:
        st.params[k] = st.params[k][keep]
        m, v = st.adam[k]
        st.adam[k] = (m[keep], v[keep])
    for k in ("max_radii2d", "xyz_grad_accum", "xyz_grad_accum_abs", "denom", "tmp_radii"):
        if st.stats.get(k) is not None:
            st.stats[k] = st.stats[k][keep]
    if st.score is not None:
        st.score = st.score[keep]


def append_new_points(st: State, new):
    if new["means3d"].shape[0] == 0:
        return
    for k in PARAMS:
        st.params[k] = np.concatenate([st.params[k], new[k]], axis=0)
        m, v = st.adam[k]
        z = np.zeros_like(new[k])
        st.adam[k] = (np.concatenate([m, z], axis=0), np.concatenate([v, z], axis=0))
    if st.stats.get("tmp_radii") is not None:
        st.stats["tmp_radii"] = np.concatenate([st.stats["tmp_radii"], new["tmp_radii"]], axis=0)
    if st.score is not None:
        st.score = np.concatenate([st.score, np.zeros(new["means3d"].shape[0], np.float32)])
    st.reset_stats()


def densify_and_clone(st: State, metric_mask, clone_filter):
    selected = metric_mask & clone_filter
    if not np.any(selected):
        return 0
    new = {k: st.params[k][selected] for k in PARAMS}
    new["tmp_radii"] = st.stats["tmp_radii"][selected]
    append_new_points(st, new)
    return int(np.sum(selected))


def densify_and_split(st: State, metric_mask, split_filter, rng, split_factor):
    selected = metric_mask & split_filter
    if selected.size < st.n:  # rows appended by a clone in the same call are not split
        selected = np.concatenate([selected, np.zeros(st.n - selected.size, bool)])
    if not np.any(selected):
        return 0, 0
    means = st.params["means3d"][selected]
    log_scales = st.params["log_scales"][selected]
    scales = np.exp(log_scales).astype(np.float32)
    rotations = st.params["rotations"][selected]
    rotmats = quat_to_rotmat(rotations)
    repeated_scales = np.repeat(scales, split_factor, axis=0)
    repeated_rotmats = np.repeat(rotmats, split_factor, axis=0)
    local_samples = rng.normal(loc=0.0, scale=repeated_scales).astype(np.float32)
    offsets = np.einsum("nij,nj->ni", repeated_rotmats, local_samples)
    repeated_means = np.repeat(means, split_factor, axis=0)
    repeated_log_scales = np.repeat(log_scales, split_factor, axis=0)
    new_scales = np.log(np.exp(repeated_log_scales) / (0.8 * float(split_factor)))
    new = {
        "means3d": (repeated_means + offsets).astype(np.float32),
        "features_dc": np.repeat(st.params["features_dc"][selected], split_factor, axis=0),
        "features_rest": np.repeat(st.params["features_rest"][selected], split_factor, axis=0),
        "opacity_logits": np.repeat(st.params["opacity_logits"][selected], split_factor, axis=0),
        "log_scales": new_scales.astype(np.float32),
        "rotations": np.repeat(rotations, split_factor, axis=0),
        "tmp_radii": np.repeat(st.stats["tmp_radii"][selected], split_factor, axis=0),
    }
    append_new_points(st, new)
    count = int(np.sum(selected))
    prune_points(st, np.concatenate([selected, np.zeros(count * split_factor, bool)]))
    return count, count * split_factor


def set_opacity_cap(st: State, cap):
    """cap_opacity_logits / reset_opacity_logits: logit(min(sigmoid(l), cap)),
    and the opacity moments restart at zero (replace_state_np, :140-154)."""
    op = sigmoid(st.params["opacity_logits"]).astype(np.float32)
    st.params["opacity_logits"] = logit(np.minimum(op, cap).astype(np.float32)).astype(np.float32)
    m, v = st.adam["opacity_logits"]
    st.adam["opacity_logits"] = (np.zeros_like(m), np.zeros_like(v))


def densify_and_prune(st: State, args, scene_extent, importance_score, rng):
    denom = np.maximum(st.stats["denom"], 1.0)
    grad_vars = st.stats["xyz_grad_accum"] / denom
    grads_abs = st.stats["xyz_grad_accum_abs"] / denom
    grad_q = np.abs(grad_vars) >= args.grad_thresh
    grad_q_abs = np.abs(grads_abs) >= args.grad_abs_thresh
    max_scale = np.max(np.exp(st.params["log_scales"]), axis=1)
    clone_q = max_scale <= args.dense * scene_extent
    split_q = max_scale > args.dense * scene_extent
    metric_mask = importance_score > args.importance_score_threshold
    clone_candidates = int(np.sum(metric_mask & clone_q & grad_q))
    split_candidates = int(np.sum(metric_mask & split_q & grad_q_abs))
    cloned = densify_and_clone(st, metric_mask, clone_q & grad_q)
    split_sources, split_children = densify_and_split(st, metric_mask, split_q & grad_q_abs, rng,
                                                      args.split_factor)
    opacities = sigmoid(st.params["opacity_logits"])
    opacity_prune = opacities < args.min_opacity
    prune = opacity_prune.copy()
    screen_prune = np.zeros_like(prune)
    if args.max_screen_size > 0:
        screen_prune = st.stats["max_radii2d"] > args.max_screen_size
        prune = prune | screen_prune
    world_prune = np.zeros_like(prune)
    if args.max_world_scale_factor > 0.0:
        world_prune = np.max(np.exp(st.params["log_scales"]), axis=1) > args.max_world_scale_factor * scene_extent
        prune = prune | world_prune
    to_remove = int(np.sum(prune))
    budget = int(args.prune_budget_factor * to_remove)
    removed = 0
    if budget > 0 and st.score is not None and st.score.size > 0:
        weights = (1.0 / (1.0e-6 + (1.0 - st.score))).astype(np.float32)
        cand = np.flatnonzero(prune)
        if cand.size > 0:
            w = weights[cand]
            w = w / max(float(np.sum(w)), 1.0e-6)
            chosen = rng.choice(cand, size=min(budget, cand.size), replace=False, p=w)
            final = np.zeros_like(prune)
            final[chosen] = True
            final &= prune
            removed = int(np.sum(final))
            prune_points(st, final)
    set_opacity_cap(st, args.opacity_cap_after_densify)
    return {"metric_hits": int(np.sum(metric_mask)), "clone_candidates": clone_candidates,
            "split_candidates": split_candidates, "cloned": cloned, "split_sources": split_sources,
            "split_children": split_children, "opacity_prune_candidates": int(np.sum(opacity_prune)),
            "screen_prune_candidates": int(np.sum(screen_prune)),
            "world_prune_candidates": int(np.sum(world_prune)), "total_prune_candidates": to_remove,
            "prune_budget": budget, "actual_removed": removed}


def final_prune(st: State, min_opacity, pruning_score, score_thresh, min_gaussians):
    opacities = sigmoid(st.params["opacity_logits"])
    opacity_mask = opacities < min_opacity
    score_mask = pruning_score > score_thresh
    prune = opacity_mask | score_mask
    total = int(prune.size)
    requested = int(np.sum(prune))
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
    removed = int(np.sum(actual))
    prune_points(st, actual)
    return {"total": total, "opacity_hits": int(np.sum(opacity_mask)), "score_hits": int(np.sum(score_mask)),
            "requested_remove": requested, "actual_remove": removed, "kept": total - removed}
