"""Pin the oracle's ensemble apply to upstream CatBoost 1.2.10 predictions.

For every end-to-end fixture, the upstream model's own trees (split features,
border values, learning-rate-scaled leaf values), flattened the way
cb_model::flatten_oblivious_f64 does (crates/cb-model/src/gpu_apply.rs:120-193),
are applied by orc_apply_oblivious (crates/cb-model/src/apply.rs:374-410) and
compared with upstream's staged approximants on the training rows, its
predictions, and its held-out NaN-mode predictions, at the reference's own
1e-5 bar (crates/cb-oracle/src/compare.rs:46-148).
"""
import numpy as np
import pytest

from golden_io import load_scenario, scenario_names
from oracle import oracle

TOL = 1e-5
FMAX = float(np.finfo(np.float32).max)


def _bias(sc):
    # the starting approximant (boosting.rs:1871); the oracle's value is pinned
    # against upstream's staged approximants by test_oracle_golden.py
    p = sc["params"]
    bins = oracle.quantize(sc["X"].T.copy(), sc["borders"])
    fit = oracle.train(bins, sc["border_counts"], sc["y"], loss=p["loss"], depth=p["depth"], iterations=1,
                       learning_rate=p["learning_rate"], l2_leaf_reg=p["l2_leaf_reg"],
                       boost_from_average=p["boost_from_average"], weights=sc.get("weights"), staged=False,
                       n_threads=1)
    return fit.bias


def _nan_above(sc):
    return np.array([len(b) > 0 and b[-1] == FMAX for b in sc["borders"]], dtype=np.uint8)


@pytest.mark.parametrize("name", scenario_names())
def test_apply_matches_upstream(name):
    sc = load_scenario(name)
    flat = oracle.flatten_oblivious(sc["split_feature"], sc["split_border"], sc["leaf_values"])
    bias = _bias(sc)
    na = _nan_above(sc)
    pred = oracle.apply_oblivious(sc["X"].T, flat, bias, na)
    if "staged" in sc:
        assert np.max(np.abs(pred - sc["staged"][-1])) <= TOL
    if "predictions" in sc:
        assert np.max(np.abs(pred - sc["predictions"])) <= TOL
    if "preds_eval" in sc:
        pe = oracle.apply_oblivious(sc["X_eval"].T, flat, bias, na)
        assert np.max(np.abs(pe - sc["preds_eval"])) <= TOL


def test_apply_edge_rules():
    X = np.array([[np.nan, -1.0, 0.5, 2.0]], dtype=np.float32)
    # one tree, one split on feature 0 at 0.0; leaves [10, 20]
    flat = (np.array([0], np.uint32), np.array([0.0]), np.array([0, 1], np.uint32),
            np.array([10.0, 20.0]), np.array([0, 2], np.uint32))
    assert oracle.apply_oblivious(X, flat, 1.0).tolist() == [11.0, 11.0, 21.0, 21.0]
    # nan_mode=Max sends NaN above every border
    assert oracle.apply_oblivious(X, flat, 1.0, np.array([1], np.uint8)).tolist() == [21.0, 11.0, 21.0, 21.0]
    # a split on a feature the batch lacks never passes
    flat2 = (np.array([5], np.uint32),) + flat[1:]
    assert oracle.apply_oblivious(X, flat2, 0.0).tolist() == [10.0] * 4
    # a tree with fewer leaves than its splits address contributes 0 there
    flat3 = flat[:3] + (np.array([10.0]), np.array([0, 1], np.uint32))
    assert oracle.apply_oblivious(X, flat3, 0.0).tolist() == [10.0, 10.0, 0.0, 0.0]
    # bias + ordered sum over trees, with -0.0 + 0.0 = +0.0 at the end
    z = oracle.apply_oblivious(X[:, :1], (np.zeros(0, np.uint32), np.zeros(0), np.array([0], np.uint32),
                                          np.zeros(0), np.array([0], np.uint32)), -0.0)
    assert z[0] == 0.0 and not np.signbit(z[0])
