"""The diagonal multi-output losses on the device arm against upstream and the oracle.

MultiClassOneVsAll, MultiLogloss and MultiCrossEntropy ride the multi-output
device arm (csrc/multi.cu): per dimension p = sigmoid(a_d), der1 = t_d - p,
der2 = -p (1 - p) (crates/cb-compute/src/loss.rs:501-560), K + 1 channel
histograms scored by the multi-dimensional score, and each dimension's Newton
leaf s1 / (-s2 + l2) solved on its own (crates/cb-train/src/boosting.rs:
8323-8420).  RMSEWithUncertainty shares the diagonal leaf with its own ders
(loss.rs:680-720), leaf sums at the tree's score shift less 2 (its ders are
unbounded), and the starting approximant [f32 mean, 0.5 ln f32 var]
(boosting.rs:1895-1914).  Trees must match the oracle's; leaf values and
staged approximants within the reference's 1e-5 bar.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "multi_output.npz")


@pytest.fixture(scope="module")
def cb():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    cb.load_library()
    return cb


def _fp(cb, **kw):
    base = dict(loss="MultiClass", depth=4, iterations=5, learning_rate=0.1, l2_leaf_reg=3.0,
                score_function="Cosine", bootstrap_type="No", subsample=0.66, bagging_temperature=1.0,
                random_seed=0, boost_from_average=False)
    base.update(kw)
    return cb.FitParams(**base)


@pytest.mark.parametrize("sc", ["multiclass_onevsall", "multilogloss", "multicrossentropy", "rmse_uncertainty"])
def test_multi_output_fixture(cb, sc):
    z = np.load(GOLDEN)
    p = json.loads(str(z[f"{sc}__params"]))
    X = z["X"]
    borders = [oracle.select_borders(X[:, f], p["border_count"], p["border_type"], "Min") for f in range(X.shape[1])]
    fp = _fp(cb, depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
             l2_leaf_reg=p["l2_leaf_reg"], score_function=p["score_function"])
    labels = z[f"{sc}__labels"]
    target = {"MultiClassOneVsAll": lambda: np.argmax(labels, axis=0),
              "RMSEWithUncertainty": lambda: labels[0]}.get(p["loss"], lambda: labels)()
    m = cb.fit_multiclass([X[:, f].copy() for f in range(X.shape[1])], borders, target, p["approx_dimension"], fp,
                          staged=True, loss=p["loss"])
    np.testing.assert_array_equal(m.split_feature, z[f"{sc}__split_feature"])
    np.testing.assert_array_equal(m.split_borders().astype(np.float32), z[f"{sc}__split_border"].astype(np.float32))
    assert np.max(np.abs(m.leaf_values - z[f"{sc}__leaf_values"])) <= TOL
    assert np.max(np.abs(m.staged - z[f"{sc}__staged"])) <= TOL


CASES = [
    dict(loss="MultiClassOneVsAll", n=20000, F=10, K=4, depth=5, boot="Bernoulli", score="Cosine", it=5, w=False),
    dict(loss="MultiClassOneVsAll", n=6000, F=6, K=3, depth=3, boot="No", score="SolarL2", it=4, w=True),
    dict(loss="MultiLogloss", n=30000, F=12, K=3, depth=6, boot="Bayesian", score="L2", it=4, w=True),
    dict(loss="MultiLogloss", n=70001, F=5, K=2, depth=8, boot="No", score="Cosine", it=3, w=False),
    dict(loss="MultiCrossEntropy", n=15000, F=8, K=5, depth=4, boot="No", score="Cosine", it=5, w=False),
    dict(loss="MultiCrossEntropy", n=8000, F=6, K=1, depth=4, boot="Bernoulli", score="L2", it=4, w=True),
    dict(loss="RMSEWithUncertainty", n=25000, F=8, K=2, depth=6, boot="No", score="L2", it=6, w=False),
    dict(loss="RMSEWithUncertainty", n=7000, F=5, K=2, depth=4, boot="No", score="Cosine", it=5, w=True),
]


def _data(case):
    rs = np.random.RandomState(case["n"] + 31 * case["K"])
    n, F, K = case["n"], case["F"], case["K"]
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.03] = np.nan
    lin = np.nan_to_num(X[:, :min(F, max(K, 2))]) @ rs.standard_normal((min(F, max(K, 2)), K))
    if case["loss"] == "MultiClassOneVsAll":
        target = np.argmax(lin + rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    elif case["loss"] == "RMSEWithUncertainty":  # heteroscedastic: the noise grows with feature 1
        target = lin[:, 0] + np.exp(0.5 * np.nan_to_num(X[:, 1])) * rs.standard_normal(n)
    elif case["loss"] == "MultiLogloss":
        target = (lin + rs.logistic(size=(n, K)) > 0).T.astype(np.float64)
    else:  # soft labels in [0, 1], the two ends included
        target = np.clip(1.0 / (1.0 + np.exp(-lin)) + rs.uniform(-0.2, 0.2, (n, K)), 0.0, 1.0).T.copy()
    w = rs.uniform(0.2, 2.0, n) if case["w"] else None
    return X, target, w


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['loss']}-K{c['K']}-{c['boot']}-d{c['depth']}-n{c['n']}")
def test_multi_output_matches_oracle(cb, case):
    X, target, w = _data(case)
    F, K = case["F"], case["K"]
    borders = [oracle.select_borders(X[:, f], 64) for f in range(F)]
    fp = _fp(cb, depth=case["depth"], iterations=case["it"], bootstrap_type=case["boot"],
             score_function=case["score"], subsample=0.66, random_seed=11)
    m = cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, target, K, fp, weights=w, staged=True,
                          loss=case["loss"])
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_multiclass(bins, [len(b) for b in borders], target, K, depth=fp.depth,
                                iterations=fp.iterations, learning_rate=fp.learning_rate,
                                l2_leaf_reg=fp.l2_leaf_reg, score_function=fp.score_function,
                                bootstrap_type=fp.bootstrap_type, subsample=fp.subsample,
                                bagging_temperature=fp.bagging_temperature, random_seed=fp.random_seed,
                                weights=w, loss=case["loss"])
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def test_multi_output_label_checks_and_declines(cb):
    from catboost_rs_b200 import CbGpuError
    rs = np.random.RandomState(5)
    n, F, K = 3000, 4, 3
    X = rs.standard_normal((n, F)).astype(np.float32)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1

    def begin(loss, k=K):
        rt = cb.B200MultiRuntime()
        ok = rt.begin_device_training_raw(loss, 3, True, 1, "Cosine", cols, borders, None, n, F, nb, 0.1, 3.0,
                                          cb.DeviceTrainConfig(), approx_dim=k)
        return rt, ok

    # one dimension is a label loss only; OneVsAll, like MultiClass, needs two classes
    rt, ok = begin("MultiClassOneVsAll", 1)
    assert not ok and rt.decline_reason
    rt, ok = begin("MultiLogloss", 1)
    assert ok
    rt.end_device_training()
    labels = (rs.uniform(size=(K, n)) < 0.5).astype(np.float64)
    for loss, bad_value in (("MultiLogloss", 0.5), ("MultiCrossEntropy", 1.25), ("MultiCrossEntropy", np.nan)):
        rt, ok = begin(loss)
        assert ok
        bad = labels.copy()
        bad[2, 7] = bad_value
        with pytest.raises(CbGpuError, match="label"):
            rt.grow_tree_on_device(None, bad, [], family=("MultiOutput", None, K))
        rt.end_device_training()
    rt, ok = begin("MultiLogloss")
    with pytest.raises(CbGpuError, match="LengthMismatch"):
        rt.grow_tree_on_device(None, labels[0], [], family=("MultiOutput", None, K))  # [n], not [K, n]
    t = rt.grow_tree_on_device(None, labels, [], family=("MultiOutput", None, K))
    assert len(t.splits) == 3 and t.leaf_values.size == 8 * K
    rt.end_device_training()
