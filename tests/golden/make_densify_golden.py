"""Generates tests/golden/densify_ref.npz by running the reference's own FastGS
densification functions (test infrastructure; run where the reference tree
exists):

    python tests/golden/make_densify_golden.py [--reference-dir DIR]

The reference densifies on the host with NumPy
(scripts/train_scanner_fastgs.py:343-795); its only MLX uses on that path are
array construction, mx.eval, mx.take / mx.concatenate / mx.zeros for the
optimizer-state surgery (:103-154) and the model getters
(scripts/train_scanner_fixed.py:505-535: mx.sigmoid, mx.exp, mx.linalg.norm).
MLX is not installable here, so this script puts a NumPy stand-in for those
calls in sys.modules["mlx"] and imports the reference's unmodified
train_scanner_fastgs.py. Its own functions then run as written:
densify_and_prune_fastgs, final_prune_fastgs, prune_points and
reset_opacity_logits, with the optimizer states of
ScannerFastGSOptimizerPolicy.

Cases (300 Gaussians, seeded; inputs and outputs stored per name):
  clone_cap    clone candidates only, no prune budget: clone + opacity cap
  prune_cap    no densification candidates: the budgeted prune (rng.choice)
               + opacity cap
  split        split candidates only (children offsets from rng.normal)
  clone_prune  clone candidates and a prune budget
  both         clone and split candidates in one call
  final_prune  final_prune_fastgs with the minimum-count path
  reset        reset_opacity_logits
  prune        prune_points of a random mask
The reference's own code raises in three of them, and the exception is
recorded with the parameters as it left them: append_new_points never resizes
state.tmp_radii (:477-507), so any prune_points after an append in the same
call fails on it (split, whose sources are pruned after the children are
appended, and clone_prune); and densify_and_split_fastgs indexes the
post-clone arrays with pre-clone masks (both). In split the failure comes
after prune_points has already applied the pruned parameters and moments,
so the recorded state is the whole split result (children appended, sources
removed), which pins the split arithmetic.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
NAMES = ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations")


def _install_mlx_stand_in() -> None:
    """NumPy behind the mlx names the densification path calls."""
    core = types.ModuleType("mlx.core")
    core.float32, core.uint32, core.int32, core.bool_ = np.float32, np.uint32, np.int32, np.bool_

    class array:  # a class: the reference also uses mx.array in annotations (mx.array | None)
        def __new__(cls, x, dtype=None):
            return np.array(x, dtype=dtype)

    core.array = array
    core.eval = lambda *a, **k: None
    core.set_cache_limit = lambda *a, **k: None
    core.take = lambda a, idx, axis=0: np.take(a, idx, axis=axis)
    core.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    core.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype)
    core.zeros_like = np.zeros_like
    core.exp = lambda x: np.exp(x).astype(np.float32)
    core.sigmoid = lambda x: (1.0 / (1.0 + np.exp(-x))).astype(np.float32)
    core.linalg = types.SimpleNamespace(norm=np.linalg.norm)
    nn = types.ModuleType("mlx.nn")

    class Module:
        def __init__(self):
            pass

    nn.Module = Module
    nn.value_and_grad = lambda *a, **k: None
    opt = types.ModuleType("mlx.optimizers")

    class Adam:
        def __init__(self, learning_rate, betas=(0.9, 0.999), eps=1e-8):
            self.learning_rate, self.betas, self.eps = learning_rate, betas, eps
            self.state = {}

    opt.Adam = Adam
    pkg = types.ModuleType("mlx")
    pkg.core, pkg.nn, pkg.optimizers = core, nn, opt
    sys.modules.update({"mlx": pkg, "mlx.core": core, "mlx.nn": nn, "mlx.optimizers": opt})


def _scene(rng, n, extent, mode):
    dense = 0.01 * extent
    p = {"means3d": rng.uniform(-1, 1, (n, 3)), "features_dc": rng.uniform(0, 1, (n, 3)),
         "features_rest": rng.normal(0, 0.05, (n, 15, 3)),
         "opacity_logits": rng.uniform(-2, 3, n), "rotations": rng.normal(0, 1, (n, 4))}
    small = np.log(dense * rng.uniform(0.1, 0.5, (n, 3)))
    big = np.log(dense * rng.uniform(2.0, 6.0, (n, 3)))
    if mode == "clone":
        ls = small
    elif mode == "split":
        ls = big
    else:
        ls = np.where((rng.random(n) < 0.5)[:, None], big, small)
    p["log_scales"] = ls
    # the first 15% are the low-opacity prune candidates; densified rows come later
    k = int(0.15 * n)
    p["opacity_logits"][:k] = rng.uniform(-9, -7, k)
    return {name: np.asarray(v, np.float32) for name, v in p.items()}, k


def _stats(rng, n, k):
    denom = rng.integers(1, 20, n).astype(np.float32)
    acc = np.where(rng.random(n) < 0.5, 1e-3, 1e-5).astype(np.float32) * denom
    acc_abs = np.where(rng.random(n) < 0.5, 5e-3, 1e-5).astype(np.float32) * denom
    acc[:k] = 0.0  # prune candidates never densify
    acc_abs[:k] = 0.0
    maxr = np.full(n, 5.0, np.float32)
    return acc, acc_abs, denom, maxr


def _model(ref, fixed, params, m, v):
    model = fixed.ScannerTrainModel(**{k: params[k].copy() for k in NAMES})
    cfg = ref.OptimizerPolicyConfig(means_lr=3e-3, dc_lr=1e-3, sh_lr=1e-3, opacity_lr=1e-3,
                                    scaling_lr=1e-3, rotation_lr=1e-3)
    pol = ref.ScannerFastGSOptimizerPolicy(cfg)
    for name in NAMES:
        opt = pol.sh_optimizer if name == "features_rest" else pol.main_optimizers[name]
        opt.state[name] = {"m": m[name].copy(), "v": v[name].copy()}
    return model, pol


def _state(ref, acc, acc_abs, denom, maxr):
    st = ref.make_densification_state(acc.size)
    st.xyz_grad_accum[:, 0] = acc
    st.xyz_grad_accum_abs[:, 0] = acc_abs
    st.denom[:, 0] = denom
    st.max_radii2d[:] = maxr
    st.tmp_radii = maxr.copy()
    return st


def _dump(out, tag, model, pol, st):
    for name in NAMES:
        out[f"{tag}_out_{name}"] = np.asarray(getattr(model, name), np.float32)
        opt = pol.sh_optimizer if name == "features_rest" else pol.main_optimizers[name]
        out[f"{tag}_out_m_{name}"] = np.asarray(opt.state[name]["m"], np.float32)
        out[f"{tag}_out_v_{name}"] = np.asarray(opt.state[name]["v"], np.float32)
    out[f"{tag}_out_acc"] = st.xyz_grad_accum[:, 0].astype(np.float32)
    out[f"{tag}_out_acc_abs"] = st.xyz_grad_accum_abs[:, 0].astype(np.float32)
    out[f"{tag}_out_denom"] = st.denom[:, 0].astype(np.float32)
    out[f"{tag}_out_max_radii"] = st.max_radii2d.astype(np.float32)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=None)
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    from oracle.build import default_reference_dir

    ref_dir = a.reference_dir or default_reference_dir()
    _install_mlx_stand_in()
    sys.path.insert(0, os.path.join(ref_dir, "scripts"))
    fixed = importlib.import_module("train_scanner_fixed")
    ref = importlib.import_module("train_scanner_fastgs")

    out = {}
    n, extent = 300, 5.0
    base = dict(grad_thresh=2.0e-4, grad_abs_thresh=1.2e-3, dense=0.01,
                importance_score_threshold=5.0, split_factor=2, min_opacity=0.005,
                max_screen_size=20.0, max_world_scale_factor=0.1, prune_budget_factor=0.5,
                opacity_cap_after_densify=0.82)
    out["extent"] = np.float32(extent)
    # tag, scene mode, densify-argument overrides, importance of the non-candidates
    cases = (("clone_cap", "clone", {"prune_budget_factor": 0.0}, 10.0),
             ("prune_cap", "both", {}, 1.0),
             ("split", "split", {"prune_budget_factor": 0.0}, 10.0),
             ("clone_prune", "clone", {}, 10.0),
             ("both", "both", {}, 10.0),
             ("final_prune", "both", None, 10.0),
             ("reset", "both", None, 10.0),
             ("prune", "both", None, 10.0))
    for ci, (tag, mode, over, imp_hi) in enumerate(cases):
        rng = np.random.default_rng(100 + ci)
        params, k = _scene(rng, n, extent, mode)
        m = {name: rng.normal(0, 1e-3, params[name].shape).astype(np.float32) for name in NAMES}
        v = {name: rng.uniform(0, 1e-6, params[name].shape).astype(np.float32) for name in NAMES}
        acc, acc_abs, denom, maxr = _stats(rng, n, k)
        importance = np.where(rng.random(n) < 0.6, imp_hi, 1.0).astype(np.float32)
        importance[:k] = 1.0
        pruning = rng.uniform(0, 0.99, n).astype(np.float32)
        for name in NAMES:
            out[f"{tag}_in_{name}"] = params[name]
            out[f"{tag}_in_m_{name}"] = m[name]
            out[f"{tag}_in_v_{name}"] = v[name]
        out[f"{tag}_in_acc"], out[f"{tag}_in_acc_abs"] = acc, acc_abs
        out[f"{tag}_in_denom"], out[f"{tag}_in_max_radii"] = denom, maxr
        out[f"{tag}_in_importance"], out[f"{tag}_in_pruning"] = importance, pruning
        seed = 1000 + ci
        out[f"{tag}_seed"] = np.int64(seed)
        dargs = None
        if over is not None:
            dargs = argparse.Namespace(**{**base, **over})
            out[f"{tag}_args"] = np.array(json.dumps(vars(dargs)))
        model, pol = _model(ref, fixed, params, m, v)
        st = _state(ref, acc, acc_abs, denom, maxr)
        res = {}
        try:
            if dargs is not None:
                res = ref.densify_and_prune_fastgs(model, st, dargs, extent, importance, pruning,
                                                   np.random.default_rng(seed), optimizer_policy=pol)
            elif tag == "final_prune":
                res = ref.final_prune_fastgs(model, st, 0.5, pruning, 0.3, 200, optimizer_policy=pol)
            elif tag == "reset":
                ref.reset_opacity_logits(model, 0.05, optimizer_policy=pol)
            else:
                mask = np.random.default_rng(seed).random(n) < 0.3
                out[f"{tag}_mask"] = mask
                ref.prune_points(model, st, mask, optimizer_policy=pol)
        except Exception as e:  # the reference's own failure, recorded as its behaviour
            out[f"{tag}_raises"] = np.array(f"{type(e).__name__}: {e}")
            print(tag, "raises", type(e).__name__, e)
            # the parameters and moments as the reference left them when it
            # raised (for a split: children appended and sources pruned; only
            # the statistics bookkeeping after that failed)
            for name in NAMES:
                out[f"{tag}_partial_{name}"] = np.asarray(getattr(model, name), np.float32)
                opt = pol.sh_optimizer if name == "features_rest" else pol.main_optimizers[name]
                out[f"{tag}_partial_m_{name}"] = np.asarray(opt.state[name]["m"], np.float32)
                out[f"{tag}_partial_v_{name}"] = np.asarray(opt.state[name]["v"], np.float32)
            continue
        out[f"{tag}_result"] = np.array(json.dumps(res))
        _dump(out, tag, model, pol, st)
        print(tag, res)
    np.savez_compressed(os.path.join(HERE, "densify_ref.npz"), **out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
