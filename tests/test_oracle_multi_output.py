"""Pin the oracle's diagonal multi-output losses to upstream.

tests/golden/multi_output.npz holds upstream CatBoost 1.2.10 fits from the
reference's crates/cb-oracle/fixtures/{multiclass_onevsall, multilogloss,
multicrossentropy}: 3 output dimensions on numeric_tiny, depth 2, 5
iterations, Newton leaves, Cosine, l2 3, lr 0.1.  All three are separable:
per dimension p = sigmoid(a_d), der1 = t_d - p, der2 = -p (1 - p)
(crates/cb-compute/src/loss.rs:501-560), and each dimension's Newton leaf is
solved on its own (crates/cb-train/src/boosting.rs:8323-8420).  The split
score is the multi-dimensional Cosine shared with MultiClass softmax.

RMSEWithUncertainty (fixture rmse_uncertainty: depth 3, 11 iterations, L2)
rides the same diagonal leaf: der1 = [diff, diff^2 prec - 1],
der2 = [-1, -2 diff^2 prec] with diff = t - a0, prec = exp(-2 a1)
(loss.rs:680-720), from the starting approximant [f32 mean, 0.5 ln f32 var]
(boosting.rs:1895-1914).  Upstream computes prec with FastExp; exp here agrees
within 3e-8 over the 11 staged approximants.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "multi_output.npz")
TOL = 1e-5
SCENARIOS = ["multiclass_onevsall", "multilogloss", "multicrossentropy", "rmse_uncertainty"]


def _load():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def _fit(d, sc, borders=None):
    p = json.loads(str(d[f"{sc}__params"]))
    X = d["X"]
    if borders is None:
        borders = [oracle.select_borders(X[:, f], p["border_count"], p["border_type"], "Min")
                   for f in range(X.shape[1])]
    bins = oracle.quantize(X.T.copy(), borders)
    labels = d[f"{sc}__labels"]
    target = {"MultiClassOneVsAll": lambda: np.argmax(labels, axis=0),
              "RMSEWithUncertainty": lambda: labels[0]}.get(p["loss"], lambda: labels)()
    fit = oracle.train_multiclass(bins, [len(b) for b in borders], target, p["approx_dimension"],
                                  depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
                                  l2_leaf_reg=p["l2_leaf_reg"], score_function=p["score_function"], loss=p["loss"])
    return borders, fit


@pytest.mark.parametrize("sc", SCENARIOS)
def test_multi_output_matches_upstream(sc):
    d = _load()
    borders, fit = _fit(d, sc)
    np.testing.assert_array_equal(fit.split_feature, d[f"{sc}__split_feature"])
    got = np.array([[borders[f][b] for f, b in zip(rf, rb)] for rf, rb in zip(fit.split_feature, fit.split_bin)])
    np.testing.assert_array_equal(got.astype(np.float32), d[f"{sc}__split_border"].astype(np.float32))
    assert np.max(np.abs(fit.leaf_values - d[f"{sc}__leaf_values"])) <= TOL
    assert np.max(np.abs(fit.staged - d[f"{sc}__staged"])) <= TOL
    # Probability: the per-dimension sigmoid (crates/cb-model/src/predict.rs:272-363);
    # RMSEWithUncertainty's fixture holds the raw [mean, log-scale] approximant
    prob = fit.final_approx if sc == "rmse_uncertainty" else 1.0 / (1.0 + np.exp(-fit.final_approx))
    assert np.max(np.abs(prob - d[f"{sc}__probabilities"])) <= TOL


def test_one_vs_all_differs_from_softmax():
    # the same classes under the coupled softmax solve give other leaves
    d = _load()
    borders, ova = _fit(d, "multiclass_onevsall")
    bins = oracle.quantize(d["X"].T.copy(), borders)
    cls = np.argmax(d["multiclass_onevsall__labels"], axis=0)
    sm = oracle.train_multiclass(bins, [len(b) for b in borders], cls, 3, depth=2, iterations=5)
    assert np.max(np.abs(sm.leaf_values - ova.leaf_values)) > 1e-3


def test_cross_entropy_on_binary_labels_equals_multilogloss():
    # one der for both losses; they differ only in the admissible targets
    d = _load()
    _, a = _fit(d, "multilogloss")
    _, b = _fit(d, "multicrossentropy")
    np.testing.assert_array_equal(a.leaf_values, b.leaf_values)


def test_soft_label_dimensions_solve_independently():
    # soft [0, 1] labels; under L2 scoring a repeated label dimension repeats
    # every leaf value and leaves the splits of the one-dimensional fit
    rs = np.random.RandomState(3)
    n = 4000
    X = rs.standard_normal((n, 3)).astype(np.float32)
    t = 1.0 / (1.0 + np.exp(-(X[:, 0] - 0.5 * X[:, 2])))
    borders = [oracle.select_borders(X[:, f], 32) for f in range(3)]
    bins = oracle.quantize(X.T.copy(), borders)
    m2 = oracle.train_multiclass(bins, [len(b) for b in borders], np.vstack([t, t]), 2, depth=3, iterations=4,
                                 loss="MultiCrossEntropy", score_function="L2")
    m1 = oracle.train_multiclass(bins, [len(b) for b in borders], t[None, :], 1, depth=3, iterations=4,
                                 loss="MultiCrossEntropy", score_function="L2")
    np.testing.assert_array_equal(m2.split_feature, m1.split_feature)
    np.testing.assert_allclose(m2.leaf_values[:, :, 0], m2.leaf_values[:, :, 1], rtol=0, atol=0)
    np.testing.assert_allclose(m2.leaf_values[:, :, 0], m1.leaf_values[:, :, 0], rtol=0, atol=1e-15)
    assert np.isfinite(m2.final_approx).all()


def test_unknown_loss_is_rejected():
    with pytest.raises(ValueError):
        oracle.train_multiclass(np.zeros((1, 4), np.uint8), [1], np.zeros(4, np.int32), 2, loss="MultiQuantile")
