"""The grouped-loss (QueryRMSE, QuerySoftMax, LambdaMart, YetiRank, YetiRankPairwise, StochasticRank, PairLogit,
PairLogitPairwise) device mode against upstream and the oracle.

The device mode (csrc/multi.cu, cbgpu_rank_begin_raw) reproduces cb-train's
grouped CPU branch: grouped ders (crates/cb-compute/src/ranking_der.rs),
PairLogit's pairwise histogram weights (boosting.rs:1761-1780), Newton leaves
and the pair-loss leaf centring (boosting.rs:2844-2880); PairLogitPairwise
scores splits with the pairwise scorer (crates/cb-compute/src/
pairwise_scoring.rs) and takes Cholesky pairwise leaves
(crates/cb-train/src/pairwise_leaves.rs).  Trees must equal the oracle's;
leaf values and staged approximants within the reference's 1e-5 bar.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ranking_corpus.npz")


@pytest.fixture(scope="module")
def cb():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    cb.load_library()
    return cb


@pytest.mark.parametrize("loss", ["QueryRMSE", "PairLogit", "PairLogitPairwise", "QuerySoftMax", "LambdaMart",
                                  "YetiRank", "StochasticRank", "YetiRankPairwise"])
def test_ranking_fixture(cb, loss):
    z = np.load(GOLDEN)
    p = json.loads(str(z[f"{loss}__params"]))
    X = z["X"]
    borders = [oracle.select_borders(X[:, f], 254, "GreedyLogSum", "Min") for f in range(X.shape[1])]
    fp = cb.FitParams(loss=loss, depth=p["depth"], iterations=p["iterations"], learning_rate=p["learning_rate"],
                      l2_leaf_reg=p["l2_leaf_reg"], random_seed=p["random_seed"], boost_from_average=False,
                      softmax_lambda=p.get("softmax_lambda", 0.01), softmax_beta=p.get("softmax_beta", 1.0),
                      lambdamart_sigma=p.get("lambdamart_sigma", 1.0), lambdamart_top=p.get("lambdamart_top", -1),
                      lambdamart_norm=p.get("lambdamart_norm", True), yeti_permutations=p.get("yeti_permutations", 10),
                      yeti_decay=p.get("yeti_decay", 0.85), srank_metric=p.get("srank_metric", "DCG"),
                      srank_sigma=p.get("srank_sigma", 1.0), srank_mu=p.get("srank_mu", 0.0),
                      srank_num_estimations=p.get("srank_num_estimations", 1))
    m = cb.fit_ranking([X[:, f].copy() for f in range(X.shape[1])], borders, z["y"], z["group_offsets"], fp,
                       pairs=z["pairs"], staged=True)
    np.testing.assert_array_equal(m.split_feature, z[f"{loss}__split_feature"])
    np.testing.assert_array_equal(m.split_borders().astype(np.float32), z[f"{loss}__split_border"].astype(np.float32))
    assert np.max(np.abs(m.leaf_values - z[f"{loss}__leaf_values"])) <= TOL
    assert np.max(np.abs(m.staged - z[f"{loss}__staged"])) <= TOL


def _ranking_data(n_groups, F, seed):
    rs = np.random.RandomState(seed)
    sizes = rs.randint(20, 121, n_groups)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    n = int(offsets[-1])
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.02] = np.nan
    score = np.nan_to_num(X[:, :3]) @ np.array([1.0, -0.5, 0.25]) + 0.5 * rs.standard_normal(n)
    y = np.zeros(n)
    pairs = []
    for g in range(n_groups):
        b, e = offsets[g], offsets[g + 1]
        q = np.quantile(score[b:e], [0.25, 0.5, 0.75])
        y[b:e] = np.digitize(score[b:e], q)
        for _ in range(2 * (e - b)):  # random within-group pairs, winner = higher relevance
            i, j = rs.randint(b, e, 2)
            if y[i] > y[j]:
                pairs.append((i, j))
            elif y[j] > y[i]:
                pairs.append((j, i))
    return X, y, offsets, np.array(pairs, dtype=np.int64)


@pytest.mark.parametrize("loss,depth,score", [("QueryRMSE", 6, "Cosine"), ("PairLogit", 5, "Cosine"),
                                              ("PairLogit", 4, "L2"), ("QuerySoftMax", 6, "Cosine")])
def test_ranking_matches_oracle(cb, loss, depth, score):
    X, y, offsets, pairs = _ranking_data(300, 10, 7 + depth)
    F = X.shape[1]
    borders = [oracle.select_borders(X[:, f], 64) for f in range(F)]
    fp = cb.FitParams(loss=loss, depth=depth, iterations=5, learning_rate=0.3, l2_leaf_reg=3.0,
                      score_function=score, boost_from_average=False)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss=loss, pairs=pairs, depth=depth,
                             iterations=5, learning_rate=0.3, l2_leaf_reg=3.0, score_function=score)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


@pytest.mark.parametrize("loss,lam,beta", [("QueryRMSE", 0.01, 1.0), ("QuerySoftMax", 0.01, 1.0),
                                           ("QuerySoftMax", 0.1, 2.0)])
def test_weighted_ranking_matches_oracle(cb, loss, lam, beta):
    # object weights with zeros: QuerySoftMax skips w <= 0 objects in its max, sums and ders
    X, y, offsets, pairs = _ranking_data(150, 8, 23)
    n, F = X.shape
    w = np.random.RandomState(5).choice([0.0, 0.5, 1.0, 2.0], size=n)
    borders = [oracle.select_borders(X[:, f], 48) for f in range(F)]
    fp = cb.FitParams(loss=loss, depth=5, iterations=4, learning_rate=0.2, l2_leaf_reg=2.0,
                      boost_from_average=False, softmax_lambda=lam, softmax_beta=beta)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, weights=w, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss=loss, depth=5, iterations=4,
                             learning_rate=0.2, l2_leaf_reg=2.0, weights=w, softmax_lambda=lam, softmax_beta=beta)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


@pytest.mark.parametrize("depth,score", [(5, "Cosine"), (4, "L2")])
def test_weighted_pairs_match_oracle(cb, depth, score):
    # PairLogit with per-pair weights (Competitor::weight): the ders scale by
    # the weight and the pairwise histogram weights sum it
    X, y, offsets, pairs = _ranking_data(200, 8, 13 + depth)
    F = X.shape[1]
    pwt = np.random.RandomState(depth).choice([0.25, 0.5, 1.0, 2.0, 3.75], size=len(pairs))
    borders = [oracle.select_borders(X[:, f], 48) for f in range(F)]
    fp = cb.FitParams(loss="PairLogit", depth=depth, iterations=4, learning_rate=0.3, l2_leaf_reg=3.0,
                      score_function=score, boost_from_average=False)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True,
                       pair_weights=pwt)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="PairLogit", pairs=pairs, depth=depth,
                             iterations=4, learning_rate=0.3, l2_leaf_reg=3.0, score_function=score,
                             pair_weights=pwt)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL
    # unit weights given explicitly are the unweighted fit
    u = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True,
                       pair_weights=np.ones(len(pairs)))
    v = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True)
    np.testing.assert_array_equal(u.staged, v.staged)


def test_weighted_pairs_rules(cb):
    from catboost_rs_b200 import CbGpuError
    X, y, offsets, pairs = _ranking_data(20, 4, 3)
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1
    w = np.full(len(pairs), 2.0)
    rt = cb.B200MultiRuntime()  # the pairwise scorer takes unit pair weights
    ok = rt.begin_ranking_raw("PairLogitPairwise", 3, True, 1, "Cosine", cols, borders, None, n, F, nb, 0.3, 3.0,
                              cb.DeviceTrainConfig(), offsets, pairs, pair_weights=w)
    assert not ok and "unit pair weights" in rt.decline_reason
    w[3] = np.nan
    with pytest.raises(CbGpuError, match="non-finite weight"):
        cb.B200MultiRuntime().begin_ranking_raw("PairLogit", 3, True, 1, "Cosine", cols, borders, None, n, F, nb,
                                                0.3, 3.0, cb.DeviceTrainConfig(), offsets, pairs, pair_weights=w)
    with pytest.raises(CbGpuError, match="one weight per pair"):
        cb.B200MultiRuntime().begin_ranking_raw("PairLogit", 3, True, 1, "Cosine", cols, borders, None, n, F, nb,
                                                0.3, 3.0, cb.DeviceTrainConfig(), offsets, pairs,
                                                pair_weights=np.ones(2))


@pytest.mark.parametrize("metric", ["MRR", "ERR", "MAP"])
def test_lambdamart_no_op_metrics_match_oracle(cb, metric):
    # the reference accepts LambdaMart's MRR / ERR / MAP and leaves every der
    # at zero (ranking_der.rs:574-581): zero leaves, the first-wins split
    X, y, offsets, pairs = _ranking_data(40, 5, 32)
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    fp = cb.FitParams(loss="LambdaMart", depth=3, iterations=2, learning_rate=0.2, l2_leaf_reg=3.0,
                      boost_from_average=False, lambdamart_metric=metric)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="LambdaMart", depth=3, iterations=2,
                             learning_rate=0.2, l2_leaf_reg=3.0, lambdamart_metric=metric)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert not np.any(m.raw_leaf_values) and not np.any(o.raw_leaf_values)
    assert np.max(np.abs(m.staged - o.staged)) == 0.0


@pytest.mark.parametrize("top,norm,sigma", [(-1, True, 1.0), (5, True, 2.0), (-1, False, 0.5), (300, True, 1.0)])
def test_lambdamart_matches_oracle(cb, top, norm, sigma):
    # groups of 20-120 documents: the per-group sort, the top cut and the norm rescale
    X, y, offsets, pairs = _ranking_data(120, 8, 31)
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 48) for f in range(F)]
    fp = cb.FitParams(loss="LambdaMart", depth=5, iterations=4, learning_rate=0.2, l2_leaf_reg=3.0,
                      boost_from_average=False, lambdamart_sigma=sigma, lambdamart_top=top, lambdamart_norm=norm)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="LambdaMart", depth=5, iterations=4,
                             learning_rate=0.2, l2_leaf_reg=3.0, lambdamart_sigma=sigma, lambdamart_top=top,
                             lambdamart_norm=norm)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def _ranking_data_sizes(sizes, F, seed, self_pair=False):
    # _ranking_data with given group sizes; pairs include repeats, and with
    # self_pair one document is its own competitor
    rs = np.random.RandomState(seed)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    n = int(offsets[-1])
    X = rs.standard_normal((n, F)).astype(np.float32)
    score = X[:, :3] @ np.array([1.0, -0.5, 0.25]) + 0.5 * rs.standard_normal(n)
    y = np.zeros(n)
    pairs = []
    for g in range(len(sizes)):
        b, e = offsets[g], offsets[g + 1]
        q = np.quantile(score[b:e], [0.25, 0.5, 0.75])
        y[b:e] = np.digitize(score[b:e], q)
        for _ in range(2 * (e - b)):
            i, j = rs.randint(b, e, 2)
            if y[i] > y[j]:
                pairs.append((i, j))
            elif y[j] > y[i]:
                pairs.append((j, i))
    if self_pair:
        pairs.insert(len(pairs) // 2, (int(offsets[1]) + 3, int(offsets[1]) + 3))
    return X, y, offsets, np.array(pairs, dtype=np.int64)


# Group sizes on both sides of the device kernels' per-group paths: the
# YetiRank derivative walks only the non-zero cells up to 128 documents and
# the dense matrix beyond; its sampler keeps a group in shared memory up to
# 256 documents (one to eight 32-document slots per lane) and in global
# scratch beyond.
BIG_GROUPS = [60, 140, 250, 300, 90, 200, 129, 257, 128, 33]


@pytest.mark.parametrize("loss", ["YetiRank", "YetiRankPairwise", "PairLogit"])
def test_large_groups_match_oracle(cb, loss):
    X, y, offsets, pairs = _ranking_data_sizes(BIG_GROUPS, 6, 91, self_pair=(loss == "PairLogit"))
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    kw = dict(yeti_permutations=4, yeti_decay=0.85) if loss.startswith("YetiRank") else {}
    fp = cb.FitParams(loss=loss, depth=4, iterations=3, learning_rate=0.3, l2_leaf_reg=1.0, random_seed=5,
                      boost_from_average=False, **kw)
    prs = pairs if loss == "PairLogit" else None
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=prs, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss=loss, pairs=prs, depth=4,
                             iterations=3, learning_rate=0.3, l2_leaf_reg=1.0, random_seed=5, **kw)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


@pytest.mark.parametrize("perms,decay,weighted", [(10, 0.85, False), (3, 0.5, True)])
def test_yetirank_matches_oracle(cb, perms, decay, weighted):
    # pairs resampled on the device every tree from the host seeder's query seeds;
    # the learning-fold approximant drives the splits, the model's the leaves
    X, y, offsets, pairs = _ranking_data(80, 8, 57)
    n, F = X.shape
    w = None
    if weighted:  # one weight per group: the group weight is the members' mean
        gw = np.random.RandomState(2).choice([0.5, 1.0, 2.0], size=offsets.size - 1)
        w = np.repeat(gw, np.diff(offsets))
    borders = [oracle.select_borders(X[:, f], 48) for f in range(F)]
    fp = cb.FitParams(loss="YetiRank", depth=5, iterations=4, learning_rate=0.3, l2_leaf_reg=1.0, random_seed=11,
                      boost_from_average=False, yeti_permutations=perms, yeti_decay=decay)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, weights=w, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="YetiRank", depth=5, iterations=4,
                             learning_rate=0.3, l2_leaf_reg=1.0, random_seed=11, weights=w,
                             yeti_permutations=perms, yeti_decay=decay)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


@pytest.mark.parametrize("depth,weighted", [(4, False), (6, True)])
def test_yetirank_pairwise_matches_oracle(cb, depth, weighted):
    # YetiRank's device resamples through the pairwise scorer with weighted
    # int64 pair statistics and Cholesky leaves (stored and learning fold)
    X, y, offsets, pairs = _ranking_data(50, 6, 61 + depth)
    n, F = X.shape
    w = None
    if weighted:
        gw = np.random.RandomState(8).choice([0.5, 1.0, 2.0], size=offsets.size - 1)
        w = np.repeat(gw, np.diff(offsets))
    borders = [oracle.select_borders(X[:, f], 24) for f in range(F)]
    fp = cb.FitParams(loss="YetiRankPairwise", depth=depth, iterations=3, learning_rate=0.3, l2_leaf_reg=1.0,
                      random_seed=5, boost_from_average=False, yeti_permutations=4)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, weights=w, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="YetiRankPairwise", depth=depth,
                             iterations=3, learning_rate=0.3, l2_leaf_reg=1.0, random_seed=5, weights=w,
                             yeti_permutations=4)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


@pytest.mark.parametrize("metric,sigma,mu,ne", [("DCG", 1.0, 0.0, 1), ("NDCG", 0.5, 0.3, 3)])
def test_stochasticrank_matches_oracle(cb, metric, sigma, mu, ne):
    # per-group Monte-Carlo noise drawn on the device from the host seeder's bases
    X, y, offsets, pairs = _ranking_data(60, 8, 71)
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 48) for f in range(F)]
    fp = cb.FitParams(loss="StochasticRank", depth=4, iterations=3, learning_rate=0.3, l2_leaf_reg=3.0,
                      random_seed=9, boost_from_average=False, srank_metric=metric, srank_sigma=sigma, srank_mu=mu,
                      srank_num_estimations=ne)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="StochasticRank", depth=4,
                             iterations=3, learning_rate=0.3, l2_leaf_reg=3.0, random_seed=9, srank_metric=metric,
                             srank_sigma=sigma, srank_mu=mu, srank_num_estimations=ne)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


# depth 3 and 6 keep every level's pair-weight system in shared memory (2P <= 64);
# depth 7 scores its last level from the global scratch slots
@pytest.mark.parametrize("depth,n_groups", [(3, 60), (6, 120), (7, 40)])
def test_pairwise_matches_oracle(cb, depth, n_groups):
    X, y, offsets, pairs = _ranking_data(n_groups, 8, 40 + depth)
    F = X.shape[1]
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    fp = cb.FitParams(loss="PairLogitPairwise", depth=depth, iterations=3, learning_rate=0.3, l2_leaf_reg=3.0,
                      boost_from_average=False)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss="PairLogitPairwise", pairs=pairs,
                             depth=depth, iterations=3, learning_rate=0.3, l2_leaf_reg=3.0)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.raw_leaf_values - o.raw_leaf_values)) <= TOL
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


EDGE_LOSSES = ["QueryRMSE", "QuerySoftMax", "LambdaMart", "YetiRank", "YetiRankPairwise", "StochasticRank",
               "PairLogit", "PairLogitPairwise"]


@pytest.mark.parametrize("loss", EDGE_LOSSES)
def test_ranking_edge_groups(cb, loss):
    # singleton groups, two-document groups, groups of equal relevance and
    # documents without pairs, against the oracle
    rs = np.random.RandomState(77)
    sizes = [1, 2, 1, 5, 1, 3, 7, 2, 1, 4, 6, 1, 8, 3]
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    n, F = int(offsets[-1]), 4
    X = rs.standard_normal((n, F)).astype(np.float32)
    y = rs.randint(0, 4, n).astype(np.float64)
    y[offsets[3]:offsets[4]] = 2.0  # a group of equal relevance
    pairs = []
    for g in range(len(sizes)):
        b, e = offsets[g], offsets[g + 1]
        for i in range(b, e):
            for j in range(b, e):
                if y[i] > y[j] and rs.uniform() < 0.7:
                    pairs.append((i, j))
    pairs = np.array(pairs, dtype=np.int64).reshape(-1, 2)
    borders = [oracle.select_borders(X[:, f], 8) for f in range(F)]
    fp = cb.FitParams(loss=loss, depth=3, iterations=3, learning_rate=0.3, l2_leaf_reg=2.0, random_seed=3,
                      boost_from_average=False, yeti_permutations=3)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp, pairs=pairs, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train_ranking(bins, [len(b) for b in borders], y, offsets, loss=loss, pairs=pairs, depth=3,
                             iterations=3, learning_rate=0.3, l2_leaf_reg=2.0, random_seed=3, yeti_permutations=3)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def test_pair_losses_without_pairs(cb):
    # PairLogit with an empty pair list: zero ders everywhere, zero leaves
    X, y, offsets, _ = _ranking_data(10, 4, 5)
    F = X.shape[1]
    borders = [oracle.select_borders(X[:, f], 8) for f in range(F)]
    fp = cb.FitParams(loss="PairLogit", depth=2, iterations=2, learning_rate=0.3, boost_from_average=False)
    m = cb.fit_ranking([X[:, f].copy() for f in range(F)], borders, y, offsets, fp,
                       pairs=np.zeros((0, 2), dtype=np.int64), staged=True)
    assert np.all(m.leaf_values == 0.0) and np.all(m.staged == 0.0)


def test_ranking_declines_and_errors(cb):
    from catboost_rs_b200 import CbGpuError
    X, y, offsets, pairs = _ranking_data(20, 4, 3)
    n, F = X.shape
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1

    def begin(loss="PairLogit", boot="No", offs=offsets, prs=pairs):
        rt = cb.B200MultiRuntime()
        cfg = cb.DeviceTrainConfig(bootstrap_type=boot)
        ok = rt.begin_ranking_raw(loss, 3, True, 1, "Cosine", cols, borders, None, n, F, nb, 0.3, 3.0, cfg, offs, prs)
        return rt, ok

    rt, ok = begin(boot="Bayesian")
    assert not ok and rt.decline_reason
    rt, ok = begin(loss="RMSE")
    assert not ok
    rt = cb.B200MultiRuntime()  # the pairwise scorer covers depth 1..8
    ok = rt.begin_ranking_raw("PairLogitPairwise", 9, True, 1, "Cosine", cols, borders, None, n, F, nb, 0.3, 3.0,
                              cb.DeviceTrainConfig(), offsets, pairs, l2_leaf_reg=3.0)
    assert not ok and "depth" in rt.decline_reason
    with pytest.raises(CbGpuError, match="sigma"):
        cb.B200MultiRuntime().begin_ranking_raw("LambdaMart", 3, True, 1, "Cosine", cols, borders, None, n, F, nb,
                                                0.3, 3.0, cb.DeviceTrainConfig(), offsets, None, lambdamart_sigma=0.0)
    with pytest.raises(CbGpuError, match="crosses group"):
        begin(prs=np.array([[0, int(offsets[1])]]))  # winner and loser in different groups
    with pytest.raises(CbGpuError, match="group offsets"):
        begin(offs=np.array([0, n - 1]))
    rt, ok = begin()
    assert ok
    t = rt.grow_tree_on_device(None, y, [], leaf_of_bytes=4)
    assert len(t.splits) == 3 and t.leaf_values.size == 8 and t.leaf_of.size == n
    rt.end_device_training()
