"""Pin the oracle's Exact leaf method (MAE / Quantile) to upstream.

The Exact leaf is each leaf's weighted alpha-quantile of the f32 residuals
t - a, with the delta adjustment (crates/cb-compute/src/leaf.rs:445-520,
CPU call boosting.rs:2561-2606); the tree structure comes from quantile_der1
(loss.rs:166-193: 0 inside |t - a| < delta, else alpha or -(1 - alpha)).
The whole fits are pinned by the e2e_quantile_alpha05_mae, e2e_quantile_alpha07
and e2e_exact_leaf_{mae,quantile07} fixtures through test_oracle_golden.py;
here the function itself meets the reference's known answers
(crates/cb-compute/src/leaf_test.rs:133-163, cb-train/src/boosting_test.rs:107-135).
"""
import numpy as np
import pytest

from golden_io import load_scenario
from oracle import oracle


def test_unweighted_median_odd_count():
    assert oracle.exact_leaf_delta([2.0, -3.0, -1.0], [1.0, 1.0, 1.0], 0.5, 1e-6) == pytest.approx(-1.0 - 1e-6, abs=1e-9)


def test_empty_leaf_is_zero():
    assert oracle.exact_leaf_delta([], [], 0.5, 1e-6) == 0.0


def test_weighted_quantile():
    assert oracle.exact_leaf_delta([5.0, 0.0], [1.0, 3.0], 0.5, 1e-6) == pytest.approx(1e-6, abs=1e-9)


def test_alpha_zero_is_min():
    assert oracle.exact_leaf_delta([5.0, -2.0, 3.0], [1.0, 1.0, 1.0], 0.0, 1e-6) == pytest.approx(-2.0, abs=1e-9)


def test_alpha_is_threaded():
    r = [1.0, 2.0, 3.0, 4.0, 5.0]
    a07 = oracle.exact_leaf_delta(r, None, 0.7, 1e-6)
    a05 = oracle.exact_leaf_delta(r, None, 0.5, 1e-6)
    assert abs(a07 - 4.0) < 1e-5 and abs(a05 - 3.0) < 1e-5


def test_exact_differs_from_gradient_on_fixture():
    # the fixture's leaves are the quantiles, not the Gradient averages
    sc = load_scenario("exact_leaf_quantile07")
    p = sc["params"]
    bins = oracle.quantize(sc["X"].T.copy(), sc["borders"])
    kw = dict(loss="Quantile", depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
              l2_leaf_reg=p["l2_leaf_reg"], score_function=p["score_function"], boost_from_average=False,
              quantile_alpha=0.7)
    ex = oracle.train(bins, sc["border_counts"], sc["y"], leaf_estimation_method="Exact", **kw)
    gr = oracle.train(bins, sc["border_counts"], sc["y"], leaf_estimation_method="Gradient", **kw)
    assert np.max(np.abs(ex.final_approx - sc["predictions"])) <= 1e-5
    assert np.max(np.abs(gr.final_approx - sc["predictions"])) > 1e-2


def test_exact_needs_a_quantile_loss():
    with pytest.raises(ValueError):
        oracle.train(np.zeros((1, 4), np.uint8), [1], np.zeros(4), loss="RMSE", leaf_estimation_method="Exact")
