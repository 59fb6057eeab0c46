"""CPU training step on the oracle (TEST INFRASTRUCTURE / CPU BASELINE ONLY).

bench.py's CPU-baseline leg and its ``--impl reference`` arm time this: one
view of the training step on the host cores -- the C oracle's forward and
backward (OpenMP over Gaussians / tiles / buckets), the L1 + D-SSIM loss and
its gradient in numpy/scipy, the activation chain and the MLX-style Adam
update of all 59 floats per Gaussian in numpy. The reference has no CPU
implementation of the path (its eval_cpu methods only zero-fill), so this
port of the same algorithm is the CPU figure.
"""
from __future__ import annotations

import os
import time

import numpy as np
from scipy.ndimage import correlate1d

from oracle.oracle import Oracle


def _window():
    e = np.exp(-((np.arange(11) - 5) ** 2) / (2 * 1.5 ** 2))
    return (e / e.sum()).astype(np.float32)


def _conv(x, w):
    y = correlate1d(x, w, axis=-1, mode="constant")
    return correlate1d(y, w, axis=-2, mode="constant")


def l1_dssim(img, tgt, w_l1=1.0, w_ssim=0.2):
    """Same definition as fgs_l1_dssim_loss; img/tgt [3, H, W]."""
    w = _window()
    C1, C2 = 0.01 ** 2, 0.03 ** 2
    mx, my = _conv(img, w), _conv(tgt, w)
    exx, eyy, exy = _conv(img * img, w), _conv(tgt * tgt, w), _conv(img * tgt, w)
    A = 2 * mx * my + C1
    B = 2 * (exy - mx * my) + C2
    Cc = mx * mx + my * my + C1
    D = (exx - mx * mx) + (eyy - my * my) + C2
    S = A * B / (Cc * D)
    n = img.size
    loss = w_l1 * np.abs(img - tgt).mean() + w_ssim * (1 - S.mean())
    d_mu = 2 * my * (B - A) / (Cc * D) - 2 * mx * S * (1 / Cc - 1 / D)
    d_exx = -S / D
    d_exy = 2 * A / (Cc * D)
    g = w_l1 / n * np.sign(img - tgt) - w_ssim / n * (_conv(d_mu, w) + 2 * img * _conv(d_exx, w)
                                                       + tgt * _conv(d_exy, w))
    return float(loss), g.astype(np.float32)


def cpu_train_step(scene, cam, target, state=None, threads=None):
    """One training step of one view on the CPU. ``state`` carries the Adam
    moments between calls. Returns (loss, seconds, state)."""
    threads = threads or os.cpu_count() or 1
    o = Oracle("gpu", threads=threads)
    t0 = time.perf_counter()
    a = scene.activated()
    ins = dict(means3d=a["means3d"], dc=a["dc"], sh=a["sh"], opacities=a["opacities"],
               scales=a["scales"], rotations=a["rotations"], viewmatrix=cam.viewmatrix,
               projmatrix=cam.projmatrix, campos=cam.campos, background=np.zeros(3, np.float32),
               viewspace_points=np.zeros((scene.n, 4), np.float32))
    f = o.forward(ins, W=cam.width, H=cam.height, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy,
                  degree=scene.sh_degree)
    img = f["out_color"].reshape(3, cam.height, cam.width)
    loss, g = l1_dssim(img, target.reshape(3, cam.height, cam.width))
    b = o.backward(f, g.reshape(3, -1))
    # activation chain (sigmoid / exp / normalise) and the flat gradient
    op = a["opacities"]
    q = scene.rotations
    qn = np.linalg.norm(q, axis=1, keepdims=True)
    dq = b["dquats"]
    dr = dq / (qn + 1e-8) - q * (np.sum(q * dq, 1, keepdims=True) / (qn * (qn + 1e-8) ** 2))
    grads = np.concatenate([b["dmeans3d"].ravel(), b["ddc"].ravel(), b["dsh"].ravel(),
                            (b["dopacities"] * op * (1 - op)).ravel(),
                            (b["dscales"] * a["scales"]).ravel(), dr.ravel()]).astype(np.float32)
    params = np.concatenate([scene.means3d.ravel(), scene.features_dc.ravel(),
                             scene.features_rest.ravel(), scene.opacity_logits.ravel(),
                             scene.log_scales.ravel(), scene.rotations.ravel()]).astype(np.float32)
    if state is None:
        state = dict(m=np.zeros_like(params), v=np.zeros_like(params))
    n = scene.n
    lr = np.empty_like(params)
    for (lo, hi), r in zip(((0, 3), (3, 6), (6, 51), (51, 52), (52, 55), (55, 59)),
                           (3e-3, 1e-3, 5e-5, 1e-3, 1e-3, 1e-3)):
        lr[lo * n:hi * n] = r
    m, v = state["m"], state["v"]
    m *= 0.9
    m += 0.1 * grads
    v *= 0.99
    v += 0.01 * grads * grads
    params -= lr * m / (np.sqrt(v) + 1e-8)
    dt = time.perf_counter() - t0
    return loss, dt, state
