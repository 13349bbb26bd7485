"""Pin the oracle's MultiClass (softmax) loop to upstream CatBoost 1.2.10.

tests/golden/multiclass_softmax.npz comes from the reference's
crates/cb-oracle/fixtures/multiclass_softmax (3 classes on numeric_tiny, depth 2,
5 iterations, Newton leaves, Cosine).  The borders are the full standalone
GreedyLogSum set (border_count 254) that the oracle's pinned border selection
produces, so every candidate upstream saw competes here too.  The bar is the
reference's 1e-5 (crates/cb-oracle/src/compare.rs:46-148); split features and
border values must be identical.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "multiclass_softmax.npz")
TOL = 1e-5


def _load():
    z = np.load(GOLDEN)
    d = {k: z[k] for k in z.files}
    d["params"] = json.loads(str(d["params"]))
    return d


def _fit(d, borders, **kw):
    p = d["params"]
    bins = oracle.quantize(d["X"].T.copy(), borders)
    args = dict(depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
                l2_leaf_reg=p["l2_leaf_reg"], score_function=p["score_function"],
                bootstrap_type=p["bootstrap_type"], random_seed=p["random_seed"], n_threads=1)
    args.update(kw)
    return oracle.train_multiclass(bins, [len(b) for b in borders], d["target_class"], p["n_classes"], **args)


def _borders(d):
    p = d["params"]
    X = d["X"]
    return [oracle.select_borders(X[:, f], p["border_count"], p["border_type"], "Min") for f in range(X.shape[1])]


def test_multiclass_matches_upstream():
    d = _load()
    borders = _borders(d)
    fit = _fit(d, borders)
    np.testing.assert_array_equal(fit.split_feature, d["split_feature"])
    got_border = np.array([[borders[f][b] for f, b in zip(rf, rb)] for rf, rb in zip(fit.split_feature, fit.split_bin)])
    np.testing.assert_array_equal(got_border.astype(np.float32), d["split_border"].astype(np.float32))
    assert np.max(np.abs(fit.leaf_values - d["leaf_values"])) <= TOL
    assert np.max(np.abs(fit.staged - d["staged"])) <= TOL
    a = fit.final_approx
    e = np.exp(a - a.max(axis=1, keepdims=True))
    assert np.max(np.abs(e / e.sum(axis=1, keepdims=True) - d["probabilities"])) <= TOL


def test_multiclass_with_the_models_own_borders():
    # the model's (training-pruned) borders give the same trees
    d = _load()
    model_borders = [np.unique(d["split_border"][d["split_feature"] == f]) for f in range(d["X"].shape[1])]
    fit = _fit(d, model_borders)
    np.testing.assert_array_equal(fit.split_feature, d["split_feature"])
    assert np.max(np.abs(fit.leaf_values - d["leaf_values"])) <= TOL


def test_newton_solve():
    rs = np.random.RandomState(0)
    K = 5
    # the summed softmax Hessian of 40 objects
    H = np.zeros((K, K))
    for _ in range(40):
        a = rs.standard_normal(K)
        p = np.exp(a - a.max())
        p /= p.sum()
        H += np.outer(p, p) - np.diag(p)
    g = rs.standard_normal(K)
    packed = np.array([H[i, j] for i in range(K) for j in range(i, K)])
    l2 = 3.0
    got = oracle.solve_symmetric_newton(g, packed, l2)
    # leaf.rs:281-340: delta = -(-(H - l2 I))^-1 (-g)
    want = -np.linalg.solve(-(H - l2 * np.eye(K)), -g)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-14)
    # an empty leaf (all-zero sums) gives zeros
    assert np.array_equal(oracle.solve_symmetric_newton(np.zeros(K), np.zeros(K * (K + 1) // 2), l2), np.zeros(K))


@pytest.mark.parametrize("boot", ["Bayesian", "Bernoulli", "MVS"])
def test_multiclass_bootstraps_are_deterministic(boot):
    rs = np.random.RandomState(4)
    n, F, K = 3000, 6, 4
    X = rs.standard_normal((n, F)).astype(np.float32)
    cls = np.argmax(X[:, :K] + 0.5 * rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    bins = oracle.quantize(X.T.copy(), borders)
    a = oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=4, iterations=4,
                                bootstrap_type=boot, subsample=0.7, random_seed=3)
    b = oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=4, iterations=4,
                                bootstrap_type=boot, subsample=0.7, random_seed=3)
    np.testing.assert_array_equal(a.split_feature, b.split_feature)
    np.testing.assert_array_equal(a.leaf_values, b.leaf_values)
    # the fit learns: training log-loss falls
    def logloss(appr):
        m = appr.max(axis=1, keepdims=True)
        lse = m[:, 0] + np.log(np.exp(appr - m).sum(axis=1))
        return float(np.mean(lse - appr[np.arange(n), cls]))
    assert logloss(a.staged[-1]) < logloss(a.staged[0]) < np.log(K)
