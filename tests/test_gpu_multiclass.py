"""The multi-output (MultiClass) device arm against upstream and the oracle.

The device arm (csrc/multi.cu) reproduces cb-train's multi-output CPU branch
(crates/cb-train/src/boosting.rs:7400-8930 at approx_dimension K): softmax
derivatives, K + 1 channel histograms, multi-dim Cosine / L2 scoring, the
trace-regularised Newton leaf solve.  Trees must match the oracle's
(crates/cb-train/src/tree.rs first-wins rule); leaf values and staged
approximants within the reference's 1e-5 bar.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "multiclass_softmax.npz")


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


def _oracle(X, cls, K, borders, fp):
    bins = oracle.quantize(X.T.copy(), borders)
    return oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=fp.depth,
                                   iterations=fp.iterations, learning_rate=fp.learning_rate,
                                   l2_leaf_reg=fp.l2_leaf_reg, score_function=fp.score_function,
                                   bootstrap_type=fp.bootstrap_type, subsample=fp.subsample,
                                   bagging_temperature=fp.bagging_temperature, random_seed=fp.random_seed)


def test_multiclass_fixture(cb):
    z = np.load(GOLDEN)
    p = json.loads(str(z["params"]))
    X = z["X"]
    borders = [oracle.select_borders(X[:, f], p["border_count"], p["border_type"], "Min") for f in range(X.shape[1])]
    fp = _fp(cb, depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
             l2_leaf_reg=p["l2_leaf_reg"], score_function=p["score_function"], random_seed=p["random_seed"])
    m = cb.fit_multiclass([X[:, f].copy() for f in range(X.shape[1])], borders, z["target_class"], p["n_classes"],
                          fp, staged=True)
    np.testing.assert_array_equal(m.split_feature, z["split_feature"])
    np.testing.assert_array_equal(m.split_borders().astype(np.float32), z["split_border"].astype(np.float32))
    assert np.max(np.abs(m.leaf_values - z["leaf_values"])) <= TOL
    assert np.max(np.abs(m.staged - z["staged"])) <= TOL


CASES = [
    dict(n=5000, F=8, K=3, depth=3, boot="No", score="Cosine", it=6),
    dict(n=30000, F=20, K=10, depth=6, boot="Bernoulli", score="Cosine", it=5),
    dict(n=20000, F=15, K=5, depth=5, boot="Bayesian", score="L2", it=5),
    dict(n=70001, F=6, K=4, depth=8, boot="No", score="Cosine", it=3),
    dict(n=6000, F=8, K=4, depth=4, boot="No", score="SolarL2", it=4),
    dict(n=6000, F=8, K=3, depth=4, boot="Bernoulli", score="SatL2", it=4),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"K{c['K']}-{c['boot']}-d{c['depth']}-n{c['n']}")
def test_multiclass_matches_oracle(cb, case):
    rs = np.random.RandomState(case["n"] + case["K"])
    n, F, K = case["n"], case["F"], case["K"]
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.03] = np.nan
    lin = np.nan_to_num(X[:, :min(F, K)]) @ rs.standard_normal((min(F, K), K))
    cls = np.argmax(lin + rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    borders = [oracle.select_borders(X[:, f], 64) for f in range(F)]
    fp = _fp(cb, depth=case["depth"], iterations=case["it"], bootstrap_type=case["boot"],
             score_function=case["score"], subsample=0.66, random_seed=7)
    m = cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, cls, K, fp, staged=True)
    o = _oracle(X, cls, K, borders, fp)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def _zipf_cats(rs, n, cards):
    # Zipf-distributed categorical ints (config 3's shape), as strings
    cols = []
    for card in cards:
        p = 1.0 / np.arange(1, card + 1) ** 1.2
        cols.append([str(v) for v in rs.choice(card, size=n, p=p / p.sum())])
    return cols


def _leaf_ids(split_feature, split_bin, allbins, F):
    # routing: floats pass on bin > border, one-hot features on bin == value
    leaf = np.zeros(allbins.shape[1], dtype=np.int64)
    for l, (f, b) in enumerate(zip(split_feature, split_bin)):
        bit = (allbins[f] == b) if f >= F else (allbins[f] > b)
        leaf |= bit.astype(np.int64) << l
    return leaf


def _assert_same_partitions(m, o, allbins, F, tol):
    """Trees equal to the oracle's up to exactly tied equivalent one-hot tests:
    once a parent leaf holds only two categories of a feature, the tests
    "== a" and "== b" partition it identically with the children swapped,
    and their scores are equal in exact arithmetic, so the last bit of the
    rounding picks between them.  Every other split must be identical; the
    rows must fall into the same parts (a one-to-one relabeling of the
    leaves) with the same leaf values, and the approximants must agree."""
    T = o.split_feature.shape[0]
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    for t in range(T):
        diff = m.split_bin[t] != o.split_bin[t]
        assert (o.split_feature[t][diff] >= F).all(), (t, m.split_bin[t], o.split_bin[t])
        lm = _leaf_ids(m.split_feature[t], m.split_bin[t], allbins, F)
        lo = _leaf_ids(o.split_feature[t], o.split_bin[t], allbins, F)
        pairs = set(zip(lm.tolist(), lo.tolist()))
        assert len({a for a, _ in pairs}) == len(pairs) == len({b for _, b in pairs}), t
        for a, b in pairs:
            assert np.max(np.abs(m.leaf_values[t, a] - o.leaf_values[t, b])) <= tol, (t, a, b)
    assert np.max(np.abs(m.staged - o.staged)) <= tol


@pytest.mark.parametrize("score,depth,F,seed", [("Cosine", 5, 6, 36), ("L2", 4, 6, 35), ("Cosine", 4, 37, 72),
                                                 ("L2", 3, 62, 73)])
def test_multiclass_one_hot_matches_oracle(cb, score, depth, F, seed):
    # one-hot categorical features: equality candidates after the floats,
    # first-seen perfect-hash bins, bootstrap No (upstream rejects draws).
    # 33 float bins against up to 200 categories: past 32 float features the
    # histogram takes two launches, the first 32 * (F // 32) float features at
    # 33 bins and the rest with the one-hot features at 200 (F = 62: 30 + 4
    # features overflow one 32-lane tile)
    rs = np.random.RandomState(seed)
    n, K = 20000, 5
    X = rs.standard_normal((n, F)).astype(np.float32)
    cats = _zipf_cats(rs, n, [5, 17, 60, 200])
    codes = np.array([[int(v) for v in c] for c in cats])
    lin = X[:, :3] @ rs.standard_normal((3, K)) + 3.0 * np.eye(K)[codes[0] % K] + 1.5 * np.eye(K)[codes[2] % K]
    cls = np.argmax(lin + rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    fp = _fp(cb, depth=depth, iterations=4, score_function=score)
    m = cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, cls, K, fp, staged=True, cat_columns=cats)
    bins = oracle.quantize(X.T.copy(), borders)
    cat_bins = np.array([oracle.perfect_hash_bins(c)[0] for c in cats])
    o = oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=depth, iterations=4,
                                learning_rate=fp.learning_rate, l2_leaf_reg=fp.l2_leaf_reg, score_function=score,
                                cat_bins_fm=cat_bins)
    _assert_same_partitions(m, o, np.concatenate([bins, cat_bins.astype(bins.dtype)]), F, TOL)
    assert (m.split_feature >= F).any()  # one-hot splits were taken
    assert np.isnan(m.split_borders()[m.split_feature >= F]).all()


def test_multiclass_one_hot_declines_bootstrap(cb):
    rs = np.random.RandomState(3)
    n, F, K = 2000, 2, 3
    X = rs.standard_normal((n, F)).astype(np.float32)
    cats = _zipf_cats(rs, n, [5])
    cls = rs.randint(0, K, n).astype(np.int32)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    with pytest.raises(RuntimeError, match="bootstrap No"):
        cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, cls, K,
                          _fp(cb, bootstrap_type="Bernoulli", iterations=1), cat_columns=cats)
    with pytest.raises(RuntimeError, match="> 255"):  # more than 256 categories
        cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, cls, K, _fp(cb, iterations=1),
                          cat_columns=[[str(i % 300) for i in range(n)]])


@pytest.mark.parametrize("case", ["depth1", "absent_class", "zero_weights", "constant_feature"])
def test_multiclass_edges(cb, case):
    # depth 1, a class no row carries, zero-weight rows, a feature without borders
    rs = np.random.RandomState(21)
    n, F, K = 3000, 5, 4
    X = rs.standard_normal((n, F)).astype(np.float32)
    cls = np.argmax(X[:, :K] + rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    w = None
    depth = 4
    if case == "depth1":
        depth = 1
    elif case == "absent_class":
        cls[cls == 2] = 1
    elif case == "zero_weights":
        w = rs.choice([0.0, 1.0, 3.0], size=n)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    if case == "constant_feature":
        X[:, 2] = 0.5
        borders[2] = np.zeros(0)
    fp = _fp(cb, depth=depth, iterations=3)
    m = cb.fit_multiclass([X[:, f].copy() for f in range(F)], borders, cls, K, fp, weights=w, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=depth, iterations=3,
                                learning_rate=fp.learning_rate, l2_leaf_reg=fp.l2_leaf_reg, weights=w)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def test_multiclass_host_sample_and_run_twice(cb):
    rs = np.random.RandomState(2)
    n, F, K = 8000, 6, 3
    X = rs.standard_normal((n, F)).astype(np.float32)
    cls = rs.randint(0, K, n).astype(np.float64)
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1
    lr = float(np.float32(0.1))

    def run(sample_from_host):
        rt = cb.B200MultiRuntime()
        cfg = cb.DeviceTrainConfig(bootstrap_type="No", sample_from_host=sample_from_host)
        assert rt.begin_device_training_raw("MultiClass", 4, True, 1, "Cosine", cols, borders, None, n, F, nb, lr,
                                            3.0, cfg, approx_dim=K)
        trees = []
        for _ in range(3):
            t = rt.grow_tree_on_device(None, cls, np.ones(n) if sample_from_host else [],
                                       family=("MultiOutput", None, K), resident_approx=True, leaf_of_bytes=2)
            trees.append((t.splits, t.leaf_values.copy(), t.leaf_of.copy()))
        a = rt.resident_approx()
        rt.end_device_training()
        return trees, a

    t1, a1 = run(False)
    t2, a2 = run(True)   # an all-ones host multiplier is the no-bootstrap fit
    t3, a3 = run(False)  # run-twice bit identity
    for (s1, l1, o1), (s2, l2, o2), (s3, l3, o3) in zip(t1, t2, t3):
        assert s1 == s2 == s3
        np.testing.assert_array_equal(l1, l2)
        np.testing.assert_array_equal(l1, l3)
        np.testing.assert_array_equal(o1, o3)
    np.testing.assert_array_equal(a1, a2)
    np.testing.assert_array_equal(a1, a3)


def test_multiclass_caller_approx_and_declines(cb):
    from catboost_rs_b200 import CbGpuError
    rs = np.random.RandomState(3)
    n, F, K = 4000, 5, 3
    X = rs.standard_normal((n, F)).astype(np.float32)
    cls = rs.randint(0, K, n).astype(np.float64)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1

    def begin(**kw):
        rt = cb.B200MultiRuntime()
        cfg = cb.DeviceTrainConfig(bootstrap_type=kw.pop("boot", "No"), world_size=kw.pop("world", 1))
        ok = rt.begin_device_training_raw(kw.pop("loss", "MultiClass"), 3, True, 1, kw.pop("score", "Cosine"), cols,
                                          borders, None, n, F, nb, 0.1, 3.0, cfg, approx_dim=kw.pop("K", K))
        return rt, ok

    for kw in (dict(boot="MVS"), dict(K=1), dict(K=17), dict(loss="RMSE"), dict(score="NewtonL2")):
        rt, ok = begin(**kw)
        assert not ok and rt.decline_reason, kw
    rt, ok = begin()
    assert ok
    # a caller-supplied approximant (dim-major) is used as given
    ak = rs.standard_normal((K, n)) * 0.1
    t = rt.grow_tree_on_device(None, cls, [], family=("MultiOutput", ak, K))
    assert len(t.splits) == 3 and t.approx_dim == K and t.leaf_values.size == 8 * K
    with pytest.raises(CbGpuError):
        rt.grow_tree_on_device(None, cls, np.ones(n), family=("MultiOutput", None, K))  # no sample_from_host
    rt.end_device_training()
    rt, ok = begin()
    bad = cls.copy()
    bad[5] = K  # not a class index
    with pytest.raises(CbGpuError, match="class index"):
        rt.grow_tree_on_device(None, bad, [], family=("MultiOutput", None, K))
    rt.end_device_training()
