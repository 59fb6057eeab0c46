"""Generates tests/golden/export_ref.npz by running the reference's own
save_as_spz (scripts/train_scanner_fixed.py:631-688) on a seeded model
(test infrastructure; run where the reference tree exists):

    python tests/golden/make_export_golden.py [--reference-dir DIR]

The spz submodule the reference packs with is absent, so a stand-in `spz`
module records the arrays the reference's function assigns to
spz.GaussianCloud (positions in the app's axis frame, raw log-scales, the
rotations conjugated by the axis change, opacity logits, dc and rest
coefficients, the SH degree) instead of packing them. The mlx, cv2 and
plyfile stand-ins are those of make_dataset_golden.py. The model's rotations
are deliberately unnormalised: the reference exports model.get_rotations
(q / (|q| + 1e-8)).
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
NAMES = ("means3d", "features_dc", "features_rest", "opacity_logits", "log_scales", "rotations")


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
    # the model getters the exporter calls (scripts/train_scanner_fixed.py:524-535)
    core = sys.modules["mlx.core"]
    core.sigmoid = lambda x: (1.0 / (1.0 + np.exp(-x))).astype(np.float32)
    core.exp = lambda x: np.exp(x).astype(np.float32)
    core.linalg = types.SimpleNamespace(norm=lambda x, axis=None, keepdims=False: np.linalg.norm(
        x, axis=axis, keepdims=keepdims).astype(np.float32))
    saved = {}
    spz = types.ModuleType("spz")

    class GaussianCloud:
        pass

    class PackOptions:
        pass

    def save_spz(cloud, opts, filename):
        saved.update({k: np.array(getattr(cloud, k)) for k in (
            "positions", "scales", "rotations", "alphas", "colors", "sh")})
        saved["sh_degree"] = np.int64(cloud.sh_degree)
        saved["antialiased"] = np.int64(bool(cloud.antialiased))
        return True

    spz.GaussianCloud, spz.PackOptions, spz.save_spz = GaussianCloud, PackOptions, save_spz
    sys.modules["spz"] = spz
    sys.path.insert(0, os.path.join(ref_dir, "scripts"))
    fixed = importlib.import_module("train_scanner_fixed")
    rng = np.random.default_rng(11)
    n = 200
    params = {"means3d": rng.normal(0, 2, (n, 3)), "features_dc": rng.normal(0, 1, (n, 3)),
              "features_rest": rng.normal(0, 0.1, (n, 15, 3)),
              "opacity_logits": rng.uniform(-4, 4, n), "log_scales": rng.uniform(-6, -1, (n, 3)),
              "rotations": rng.normal(0, 1, (n, 4)) * rng.uniform(0.5, 2.0, (n, 1))}
    params = {k: np.asarray(v, np.float32) for k, v in params.items()}
    model = fixed.ScannerTrainModel(**{k: params[k].copy() for k in NAMES})
    assert fixed.save_as_spz("unused.spz", model, 3)
    out = {f"in/{k}": v for k, v in params.items()}
    out.update({f"cloud/{k}": v for k, v in saved.items()})
    path = os.path.join(HERE, "export_ref.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
