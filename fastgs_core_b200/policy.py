"""The FastGS training driver around Trainer: the optimiser policy of the
reference (ScannerFastGSOptimizerPolicy, scripts/train_scanner_fastgs.py:38-183)
and its training loop's schedule (:968-1100): the position learning-rate
decay, the optimiser cadence, staged parameter groups, the SH-degree ramp,
view sampling without replacement, densification with FastGS scores, opacity
resets and the final prune window.

The loss follows the reference's: mean squared error up to step mse_until
(its --mse-until, :824, 980), then the Trainer's L1 (the reference's is plain
L1; the Trainer adds w_ssim * D-SSIM, 0 gives the reference's).

Differences from the reference loop, by design: one render per step (its
viewspace gradient feeds the densification statistics directly, where the
reference renders a second time); best-image saving and logging are left to
the caller.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import densify as D
from .train import LearningRates, Trainer


def get_expon_lr_func(lr_init: float, lr_final: float, lr_delay_steps: int = 0,
                      lr_delay_mult: float = 1.0, max_steps: int = 1000000):
    """Log-linear decay with an optional sine-shaped delay
    (scripts/train_scanner_fastgs.py:54-74)."""

    def helper(step: int) -> float:
        if step < 0 or (lr_init == 0.0 and lr_final == 0.0):
            return 0.0
        if lr_delay_steps > 0:
            delay_rate = lr_delay_mult + (1.0 - lr_delay_mult) * math.sin(
                0.5 * math.pi * min(max(step / lr_delay_steps, 0.0), 1.0))
        else:
            delay_rate = 1.0
        t = min(max(step / max_steps, 0.0), 1.0)
        return delay_rate * math.exp(math.log(lr_init) * (1.0 - t) + math.log(lr_final) * t)

    return helper


@dataclass
class OptimizerPolicyConfig:
    """scripts/train_scanner_fastgs.py:38-51 (defaults of its command line)."""
    means_lr: float = 3e-3
    dc_lr: float = 1e-3
    sh_lr: float = 1e-3
    opacity_lr: float = 1e-3
    scaling_lr: float = 1e-3
    rotation_lr: float = 1e-3
    position_lr_init: float | None = None
    position_lr_final: float = 1.6e-6
    position_lr_delay_mult: float = 0.01
    position_lr_max_steps: int = 30000
    spatial_lr_scale: float = 1.0
    betas: tuple = (0.9, 0.99)
    sh_lr_divisor: float = 20.0


class OptimizerPolicy:
    """ScannerFastGSOptimizerPolicy (:77-183): per-group learning rates, the
    means schedule and the cadence at which groups step."""

    def __init__(self, cfg: OptimizerPolicyConfig):
        self.cfg = cfg
        xyz_init = cfg.position_lr_init if cfg.position_lr_init is not None else cfg.means_lr
        self.xyz_scheduler = get_expon_lr_func(
            lr_init=xyz_init * cfg.spatial_lr_scale,
            lr_final=cfg.position_lr_final * cfg.spatial_lr_scale,
            lr_delay_mult=cfg.position_lr_delay_mult,
            max_steps=cfg.position_lr_max_steps)

    @staticmethod
    def should_step_main(iteration: int) -> bool:
        if iteration <= 15000:
            return True
        if iteration <= 20000:
            return iteration % 32 == 0
        return iteration % 64 == 0

    @staticmethod
    def should_step_sh(iteration: int) -> bool:
        if iteration <= 15000:
            return iteration % 16 == 0
        if iteration <= 20000:
            return iteration % 32 == 0
        return iteration % 64 == 0

    def learning_rates(self, iteration: int, frozen: tuple = ()) -> LearningRates:
        """The step's rates; -1 marks a group that does not step (cadence, or
        a group named in `frozen`: names means, dc, rest, opacity, scales,
        rotations)."""
        c = self.cfg
        main = self.should_step_main(iteration)
        lr = LearningRates(
            means=self.xyz_scheduler(iteration) if main else -1.0,
            dc=c.dc_lr if main else -1.0,
            rest=c.sh_lr / c.sh_lr_divisor if self.should_step_sh(iteration) else -1.0,
            opacity=c.opacity_lr if main else -1.0,
            scales=c.scaling_lr if main else -1.0,
            rotations=c.rotation_lr if main else -1.0)
        for name in frozen:
            setattr(lr, name, -1.0)
        return lr


@dataclass
class DriverConfig:
    """The training loop's schedule (scripts/train_scanner_fastgs.py:820-849)."""
    sh_degree: int = 3
    sh_degree_interval: int = 1000
    mse_until: int = 600
    stage_color_steps: int = 0
    stage_means_steps: int = 0
    stage_scales_steps: int = 0
    stage_rotations_steps: int = 0
    densify_from_step: int = 500
    densify_until_step: int = 15000
    densification_interval: int = 500
    opacity_reset_interval: int = 3000
    opacity_reset_value: float = 0.82
    loss_thresh: float = 0.06
    densify_camera_sample: int = 10
    final_prune_min_opacity: float = 0.1
    final_prune_start: int = 15000
    final_prune_end: int = 30000
    final_prune_interval: int = 3000
    final_prune_score_thresh: float = 0.9
    final_prune_min_gaussians: int = 64
    densify: D.DensifyArgs = field(default_factory=D.DensifyArgs)


def compute_scene_extent(points: np.ndarray) -> float:
    """compute_scene_extent (:212-216)."""
    return max(float(np.linalg.norm(points.max(axis=0) - points.min(axis=0))), 1.0e-6)


def sample_camera_indices(rng, num_cameras: int, sample_count: int) -> np.ndarray:
    """sample_camera_indices (:262-265)."""
    return rng.choice(num_cameras, size=min(sample_count, num_cameras), replace=False)


class FastGSDriver:
    """Steps a Trainer through the reference's schedule. cameras: the
    training views; targets: their [3, H*W] float32 device images. With a
    data-parallel Trainer every rank runs its own driver with the same seed:
    each step renders one view per rank, and the densification and pruning
    decisions are the same on every rank."""

    def __init__(self, trainer: Trainer, cameras, targets, cfg: DriverConfig | None = None,
                 policy: OptimizerPolicy | None = None, seed: int = 42,
                 scene_extent: float | None = None):
        self.tr = trainer
        self.cameras, self.targets = cameras, targets
        self.cfg = cfg or DriverConfig()
        self.policy = policy or OptimizerPolicy(OptimizerPolicyConfig())
        self.rng = np.random.default_rng(seed)
        if scene_extent is None:
            n = trainer.n
            scene_extent = compute_scene_extent(trainer.params[:3 * n].view(n, 3).cpu().numpy())
        self.scene_extent = scene_extent
        self.step_index = 0
        self.active_sh_degree = 0
        self.viewpoint_stack: list[int] = []
        self.log: list[dict] = []

    def state_dict(self) -> dict:
        """The Trainer's state plus the driver's: step, SH degree, view stack
        and the generator's state (a resumed run draws the same views and
        makes the same densification choices)."""
        return {"trainer": self.tr.state_dict(), "step_index": self.step_index,
                "active_sh_degree": self.active_sh_degree,
                "viewpoint_stack": list(self.viewpoint_stack),
                "rng": self.rng.bit_generator.state, "scene_extent": self.scene_extent}

    def load_state_dict(self, state: dict) -> None:
        self.tr.load_state_dict(state["trainer"])
        self.step_index = int(state["step_index"])
        self.active_sh_degree = int(state["active_sh_degree"])
        self.viewpoint_stack = list(state["viewpoint_stack"])
        self.rng.bit_generator.state = state["rng"]
        self.scene_extent = float(state["scene_extent"])

    def _frozen(self, step: int) -> tuple:
        c = self.cfg
        frozen = []
        if step <= c.stage_color_steps:
            frozen += ["dc", "rest"]
        if step <= c.stage_means_steps:
            frozen.append("means")
        if step <= c.stage_scales_steps:
            frozen.append("scales")
        if step <= c.stage_rotations_steps:
            frozen.append("rotations")
        return tuple(frozen)

    def step(self, loss_out=None) -> dict:
        """One iteration; returns what happened (view, densify / prune
        statistics when they ran)."""
        c, tr = self.cfg, self.tr
        self.step_index += 1
        step = self.step_index
        tr.lrs = self.policy.learning_rates(step, self._frozen(step))
        if step % c.sh_degree_interval == 0:
            self.active_sh_degree = min(self.active_sh_degree + 1, c.sh_degree)
        tr.sh_degree = self.active_sh_degree
        tr.loss_mode = "l1_dssim" if step > c.mse_until else "mse"
        # one view per rank and step, drawn without replacement (every rank
        # draws the same ones from its equally seeded generator)
        views = []
        for _ in range(tr.world):
            if not self.viewpoint_stack:
                self.viewpoint_stack = list(range(len(self.cameras)))
            views.append(self.viewpoint_stack.pop(int(self.rng.integers(0, len(self.viewpoint_stack)))))
        tr.step([self.cameras[i] for i in views], [self.targets[i] for i in views], loss_out=loss_out)
        idx = views[0] if len(views) == 1 else views
        out = {"step": step, "view": idx, "sh_degree": self.active_sh_degree, "points": tr.n}
        if step < c.densify_until_step:
            if step > c.densify_from_step and step % c.densification_interval == 0:
                ids = sample_camera_indices(self.rng, len(self.cameras), c.densify_camera_sample)
                imp, pruning = D.compute_gaussian_scores_fastgs(tr, self.cameras, self.targets, ids,
                                                                c.loss_thresh, True)
                out["densify"] = D.densify_and_prune_fastgs(tr, c.densify, self.scene_extent, imp,
                                                            pruning, self.rng)
            if step % c.opacity_reset_interval == 0:
                D.reset_opacity_logits(tr, c.opacity_reset_value)
                out["opacity_reset"] = c.opacity_reset_value
        if (step % c.final_prune_interval == 0 and c.final_prune_start < step < c.final_prune_end):
            ids = sample_camera_indices(self.rng, len(self.cameras), c.densify_camera_sample)
            _, pruning = D.compute_gaussian_scores_fastgs(tr, self.cameras, self.targets, ids,
                                                          c.loss_thresh, False)
            out["final_prune"] = D.final_prune_fastgs(tr, c.final_prune_min_opacity, pruning,
                                                      c.final_prune_score_thresh,
                                                      c.final_prune_min_gaussians)
        out["points_after"] = tr.n
        self.log.append(out)
        return out
