"""The CPU densification checker (oracle/densify_ref.py) against fixtures made
by running the reference's own FastGS densification functions
(tests/golden/make_densify_golden.py, scripts/train_scanner_fastgs.py:470-795).

Where the reference completes (clone + cap, budgeted prune + cap, final
prune, opacity reset, prune) the checker must reproduce its parameters,
Adam moments and statistics. Where the reference raises (a split, a clone
followed by a prune, clone and split in one call) the fixture records the
exception and the parameters and moments as the reference left them; for a
split that is the whole split result, which the checker must reproduce from
the same generator."""
import json
import os

import numpy as np
import pytest

from oracle import densify_ref as R

Z = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "densify_ref.npz")))
NAMES = R.PARAMS


def state(tag, with_score=True):
    params = {k: Z[f"{tag}_in_{k}"] for k in NAMES}
    adam = {k: (Z[f"{tag}_in_m_{k}"], Z[f"{tag}_in_v_{k}"]) for k in NAMES}
    stats = {"xyz_grad_accum": Z[f"{tag}_in_acc"], "xyz_grad_accum_abs": Z[f"{tag}_in_acc_abs"],
             "denom": Z[f"{tag}_in_denom"], "max_radii2d": Z[f"{tag}_in_max_radii"],
             "tmp_radii": Z[f"{tag}_in_max_radii"]}
    return R.State(params, adam, stats, Z[f"{tag}_in_pruning"] if with_score else None)


def args(tag):
    class A:
        pass

    a = A()
    for k, v in json.loads(str(Z[f"{tag}_args"])).items():
        setattr(a, k, v)
    return a


def check_outputs(st, tag, approx=()):
    for k in NAMES:
        want = Z[f"{tag}_out_{k}"]
        if k in approx:
            np.testing.assert_allclose(st.params[k], want, rtol=1e-6, atol=1e-7, err_msg=k)
        else:
            assert np.array_equal(st.params[k], want), k
        assert np.array_equal(st.adam[k][0], Z[f"{tag}_out_m_{k}"]), k
        assert np.array_equal(st.adam[k][1], Z[f"{tag}_out_v_{k}"]), k
    for k, zk in (("xyz_grad_accum", "acc"), ("xyz_grad_accum_abs", "acc_abs"), ("denom", "denom"),
                  ("max_radii2d", "max_radii")):
        assert np.array_equal(st.stats[k], Z[f"{tag}_out_{zk}"]), k


@pytest.mark.parametrize("tag", ["clone_cap", "prune_cap"])
def test_densify_and_prune_matches_reference(tag):
    st = state(tag)
    got = R.densify_and_prune(st, args(tag), float(Z["extent"]), Z[f"{tag}_in_importance"],
                              np.random.default_rng(int(Z[f"{tag}_seed"])))
    assert got == json.loads(str(Z[f"{tag}_result"]))
    assert got["cloned"] + got["actual_removed"] > 0
    check_outputs(st, tag, approx=("opacity_logits",))


def test_final_prune_matches_reference():
    st = state("final_prune", with_score=False)
    got = R.final_prune(st, 0.5, Z["final_prune_in_pruning"], 0.3, 200)
    assert got == json.loads(str(Z["final_prune_result"]))
    check_outputs(st, "final_prune")


def test_reset_and_prune_match_reference():
    st = state("reset")
    R.set_opacity_cap(st, 0.05)
    check_outputs(st, "reset", approx=("opacity_logits",))
    st = state("prune")
    R.prune_points(st, Z["prune_mask"])
    check_outputs(st, "prune")


def test_split_matches_reference():
    """The reference raises in the statistics bookkeeping after its split has
    already been applied (append_new_points does not resize tmp_radii, which
    prune_points then indexes); the parameters and moments it left are the
    whole split result, and the checker's split must reproduce them from the
    same generator."""
    assert str(Z["split_raises"]).startswith("IndexError")
    st = state("split")
    n = st.n
    a = args("split")
    denom = np.maximum(st.stats["denom"], 1.0)
    q_abs = np.abs(st.stats["xyz_grad_accum_abs"] / denom) >= a.grad_abs_thresh
    max_scale = np.max(np.exp(st.params["log_scales"]), axis=1)
    metric = Z["split_in_importance"] > a.importance_score_threshold
    split_filter = (max_scale > a.dense * float(Z["extent"])) & q_abs
    rng = np.random.default_rng(int(Z["split_seed"]))
    # every scale is above the clone bound: the clone step selects nothing
    count, children = R.densify_and_split(st, metric, split_filter, rng, a.split_factor)
    assert count == int((metric & split_filter).sum()) > 0 and children == 2 * count
    assert st.n == n + count
    for k in NAMES:
        want = Z[f"split_partial_{k}"]
        if k in ("means3d", "log_scales"):
            np.testing.assert_allclose(st.params[k], want, rtol=1e-6, atol=1e-7, err_msg=k)
        else:
            assert np.array_equal(st.params[k], want), k
        assert np.array_equal(st.adam[k][0], Z[f"split_partial_m_{k}"]), k
        assert np.array_equal(st.adam[k][1], Z[f"split_partial_v_{k}"]), k


@pytest.mark.parametrize("tag", ["clone_prune", "both"])
def test_reference_failures_recorded(tag):
    """The two other reference failures: recorded, and resolved by the
    checker (and the GPU path) as the original 3DGS does."""
    assert str(Z[f"{tag}_raises"]).startswith("IndexError")
    st = state(tag)
    got = R.densify_and_prune(st, args(tag), float(Z["extent"]), Z[f"{tag}_in_importance"],
                              np.random.default_rng(int(Z[f"{tag}_seed"])))
    assert got["cloned"] > 0
    assert st.n == Z[f"{tag}_in_means3d"].shape[0] + got["cloned"] + got["split_children"] \
        - got["split_sources"] - got["actual_removed"]
