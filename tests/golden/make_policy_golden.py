"""Generates tests/golden/policy_ref.npz from the reference's own optimiser
policy (test infrastructure; run where the reference tree exists):

    python tests/golden/make_policy_golden.py [--reference-dir DIR]

For each sampled iteration the reference's training loop calls
ScannerFastGSOptimizerPolicy.update_learning_rate(iteration) and then
apply_gradients(model, grads, iteration)
(scripts/train_scanner_fastgs.py:77-183). A stand-in mlx Adam records which
optimisers update and at which learning rate; the fixture stores, per
iteration, the rate of each group (means, dc, rest, opacity, scales,
rotations) or -1 where the group does not step. Two configurations: the
trainer's defaults and one with a separate initial position rate and a
spatial scale. The mlx, cv2 and plyfile stand-ins are those of
make_dataset_golden.py.
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
GROUPS = (("means3d", "main"), ("features_dc", "main"), ("features_rest", "sh"),
          ("opacity_logits", "main"), ("log_scales", "main"), ("rotations", "main"))
CONFIGS = {
    "default": dict(means_lr=1.6e-4, dc_lr=2.5e-3, sh_lr=2.5e-3, opacity_lr=2.5e-2,
                    scaling_lr=5e-3, rotation_lr=1e-3),
    "scaled": dict(means_lr=1.6e-4, dc_lr=1e-3, sh_lr=1e-3, opacity_lr=5e-2, scaling_lr=1e-3,
                   rotation_lr=2e-3, position_lr_init=3e-4, position_lr_final=2e-6,
                   position_lr_delay_mult=0.05, position_lr_max_steps=20000, spatial_lr_scale=2.5),
}


def iterations() -> np.ndarray:
    it = set(range(0, 1001)) | set(range(1000, 36000, 7))
    for b in (15000, 20000, 30000):
        it |= set(range(b - 70, b + 71))
    return np.array(sorted(it), np.int64)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=None)
    a = ap.parse_args()
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    from make_dataset_golden import _install_stand_ins
    from oracle.build import default_reference_dir

    ref_dir = a.reference_dir or default_reference_dir()
    _install_stand_ins()
    log = []

    class Adam:
        def __init__(self, learning_rate, betas=(0.9, 0.999), eps=1e-8):
            self.learning_rate = learning_rate
            self.state = {}

        def update(self, model, grads):
            for name in grads:
                log.append((name, float(self.learning_rate)))

    sys.modules["mlx.optimizers"].Adam = Adam
    sys.path.insert(0, os.path.join(ref_dir, "scripts"))
    ref = importlib.import_module("train_scanner_fastgs")
    its = iterations()
    out = {"iterations": its}
    grads = {name: np.zeros(1, np.float32) for name, _ in GROUPS}
    for tag, kw in CONFIGS.items():
        pol = ref.ScannerFastGSOptimizerPolicy(ref.OptimizerPolicyConfig(**kw))
        lrs = np.full((len(its), len(GROUPS)), -1.0)
        for r, it in enumerate(its):
            log.clear()
            pol.update_learning_rate(int(it))
            pol.apply_gradients(None, grads, int(it))
            for name, lr in log:
                lrs[r, [g for g, _ in GROUPS].index(name)] = lr
        out[f"{tag}/lrs"] = lrs
    path = os.path.join(HERE, "policy_ref.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
