"""The training driver's optimiser policy and schedule (host logic; no GPU)."""
import math

import numpy as np

from fastgs_core_b200.policy import (OptimizerPolicy, OptimizerPolicyConfig, get_expon_lr_func,
                                     sample_camera_indices)


def test_expon_lr_schedule():
    f = get_expon_lr_func(3e-3, 1.6e-6, 0, 0.01, 30000)
    assert math.isclose(f(0), 3e-3)
    assert math.isclose(f(30000), 1.6e-6)
    assert math.isclose(f(60000), 1.6e-6)  # clamped past max_steps
    mid = math.exp(0.5 * (math.log(3e-3) + math.log(1.6e-6)))
    assert math.isclose(f(15000), mid)
    assert f(-1) == 0.0
    g = get_expon_lr_func(1.0, 1.0, lr_delay_steps=100, lr_delay_mult=0.01, max_steps=1000)
    assert math.isclose(g(0), 0.01)
    assert math.isclose(g(100), 1.0)


def test_cadence_and_frozen_groups():
    pol = OptimizerPolicy(OptimizerPolicyConfig())
    lr = pol.learning_rates(1)
    assert lr.rest == -1.0 and lr.dc == 1e-3 and lr.means > 0  # SH steps every 16th iteration
    assert pol.learning_rates(16).rest == 1e-3 / 20.0
    lr = pol.learning_rates(15001)
    assert lr.means == -1.0 and lr.rest == -1.0          # main every 32nd past 15000
    assert pol.learning_rates(15010).means == -1.0
    assert pol.learning_rates(15040).means > 0           # 15040 = 470 * 32
    assert pol.learning_rates(20040).means == -1.0       # every 64th past 20000
    assert pol.learning_rates(20096).means > 0
    lr = pol.learning_rates(16, frozen=("dc", "rest"))
    assert lr.dc == -1.0 and lr.rest == -1.0 and lr.opacity == 1e-3


def test_sample_camera_indices_matches_numpy():
    a = sample_camera_indices(np.random.default_rng(3), 20, 10)
    b = np.random.default_rng(3).choice(20, size=10, replace=False)
    assert np.array_equal(a, b)
    assert sample_camera_indices(np.random.default_rng(3), 4, 10).size == 4


def test_learning_rates_match_reference_policy():
    """OptimizerPolicy.learning_rates against the reference's own
    ScannerFastGSOptimizerPolicy (update_learning_rate + apply_gradients,
    recorded by tests/golden/make_policy_golden.py) over sampled iterations
    0..36000 in two configurations: every group's rate, -1 where it does not
    step."""
    import os

    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_policy_golden import CONFIGS

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "policy_ref.npz"))
    for tag, kw in CONFIGS.items():
        pol = OptimizerPolicy(OptimizerPolicyConfig(**kw))
        want = z[f"{tag}/lrs"]
        for r, it in enumerate(z["iterations"]):
            lr = pol.learning_rates(int(it))
            got = [lr.means, lr.dc, lr.rest, lr.opacity, lr.scales, lr.rotations]
            np.testing.assert_allclose(got, want[r], rtol=1e-12, atol=0, err_msg=f"{tag} {it}")
