"""Pin the oracle's grouped-loss loop (QueryRMSE, PairLogit, PairLogitPairwise, QuerySoftMax, LambdaMart, YetiRank,
YetiRankPairwise, StochasticRank) to upstream.

tests/golden/ranking_corpus.npz comes from the reference's frozen ranking
corpus (crates/cb-oracle/fixtures/ranking_corpus: 12 objects in 5 contiguous
groups, 7 explicit pairs, depth 2, 5 iterations, lr 0.3), which the
reference's own ranking oracle tests train against.  QuerySoftMax takes a
per-group softmax der (crates/cb-compute/src/ranking_der.rs:247-320) and
Gradient leaves (the fixture's leaf_estimation_method); LambdaMart the NDCG
lambda ders of a stable approx-descending sort (ranking_der.rs:482-628) with
Newton leaves; YetiRank pairs sampled per tree and phase from TFastRng64
query seeds (crates/cb-train/src/yetirank.rs) with separate learning-fold and
model approximants (boosting.rs:4997-5060, 7347-7420, 8070-8200, 8787-8880);
YetiRankPairwise the same sampled pairs, weighted, through the pairwise
scorer and Cholesky leaves; StochasticRank's Monte-Carlo DCG ders with the same seeder's recalc bases
(ranking_der.rs:640-1000, boosting.rs:5065-5100).
PairLogitPairwise scores
splits with the pairwise statistics and a per-candidate Cholesky solve
(crates/cb-compute/src/pairwise_scoring.rs) and takes its leaves from the
pairwise Cholesky system (crates/cb-train/src/pairwise_leaves.rs).  Trees are compared
both with the full standalone GreedyLogSum border set (border_count 254) and
with the model's own borders; leaf values and staged approximants at the
reference's 1e-5 bar (crates/cb-oracle/src/compare.rs:46-148).
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ranking_corpus.npz")
TOL = 1e-5


def _load():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def _fit(d, loss, borders, **kw):
    p = json.loads(str(d[f"{loss}__params"]))
    bins = oracle.quantize(d["X"].T.copy(), borders)
    args = dict(loss=loss, pairs=d["pairs"], depth=p["depth"], iterations=p["iterations"],
                learning_rate=p["learning_rate"], l2_leaf_reg=p["l2_leaf_reg"], random_seed=p["random_seed"])
    if loss == "QuerySoftMax":
        assert p["leaf_estimation_method"] == "Gradient"
        args.update(softmax_lambda=p["softmax_lambda"], softmax_beta=p["softmax_beta"])
    if loss == "StochasticRank":
        assert p["leaf_estimation_method"] == "Gradient"
        args.update(srank_metric=p["srank_metric"], srank_sigma=p["srank_sigma"], srank_mu=p["srank_mu"],
                    srank_num_estimations=p["srank_num_estimations"])
    if loss in ("YetiRank", "YetiRankPairwise"):
        args.update(yeti_permutations=p["yeti_permutations"], yeti_decay=p["yeti_decay"])
    if loss == "LambdaMart":
        assert p["leaf_estimation_method"] == "Newton" and p["lambdamart_metric"] == "NDCG"
        args.update(lambdamart_sigma=p["lambdamart_sigma"], lambdamart_top=p["lambdamart_top"],
                    lambdamart_norm=p["lambdamart_norm"])
    args.update(kw)
    return oracle.train_ranking(bins, [len(b) for b in borders], d["y"], d["group_offsets"], **args)


@pytest.mark.parametrize("loss", ["QueryRMSE", "PairLogit", "PairLogitPairwise", "QuerySoftMax", "LambdaMart",
                                  "YetiRank", "StochasticRank", "YetiRankPairwise"])
@pytest.mark.parametrize("border_set", ["full", "model"])
def test_ranking_matches_upstream(loss, border_set):
    d = _load()
    X = d["X"]
    sf, sv = d[f"{loss}__split_feature"], d[f"{loss}__split_border"]
    if border_set == "full":
        borders = [oracle.select_borders(X[:, f], 254, "GreedyLogSum", "Min") for f in range(X.shape[1])]
    else:
        borders = [np.unique(sv[sf == f]) for f in range(X.shape[1])]
    fit = _fit(d, loss, borders)
    np.testing.assert_array_equal(fit.split_feature, sf)
    got = np.array([[borders[f][b] for f, b in zip(rf, rb)] for rf, rb in zip(fit.split_feature, fit.split_bin)])
    np.testing.assert_array_equal(got.astype(np.float32), sv.astype(np.float32))
    assert np.max(np.abs(fit.leaf_values - d[f"{loss}__leaf_values"])) <= TOL
    assert np.max(np.abs(fit.staged - d[f"{loss}__staged"])) <= TOL


def test_pairlogit_leaves_are_centred():
    # normalize_leaf_values: the document-weighted mean of a PairLogit tree's
    # (pre-learning-rate) leaf values is zero; QueryRMSE leaves are not centred
    d = _load()
    X = d["X"]
    borders = [oracle.select_borders(X[:, f], 254, "GreedyLogSum", "Min") for f in range(X.shape[1])]
    fit = _fit(d, "PairLogit", borders, iterations=3)
    bins = oracle.quantize(X.T.copy(), borders)
    for t in range(3):
        leaf = np.zeros(X.shape[0], dtype=np.int64)
        for l, (f, b) in enumerate(zip(fit.split_feature[t], fit.split_bin[t])):
            leaf |= (bins[f].astype(np.int64) > b).astype(np.int64) << l
        cnt = np.bincount(leaf, minlength=fit.leaf_values.shape[1])
        assert abs(float(np.dot(fit.leaf_values[t], cnt))) < 1e-12
        assert np.any(fit.raw_leaf_values[t] != 0)


def test_group_offsets_validated():
    d = _load()
    X = d["X"]
    borders = [oracle.select_borders(X[:, f], 8) for f in range(X.shape[1])]
    bins = oracle.quantize(X.T.copy(), borders)
    with pytest.raises(RuntimeError):
        oracle.train_ranking(bins, [len(b) for b in borders], d["y"], np.array([0, 5]), loss="QueryRMSE", depth=2,
                             iterations=1)


def test_yetirank_sampler_matches_instrumented_log():
    # one 3-document group, raw approx [0.5, -0.3, 0.1], relevances [2, 0, 1],
    # 10 permutations, decay 0.85, random_seed 0 (yetirank_oracle_test.rs:213-260)
    d = _load()
    seed = oracle.yeti_query_seeds(0, 1)
    np.testing.assert_array_equal(seed, d["yeti_gt_query_seed"])
    got = oracle.yeti_sample_pairs([0.5, -0.3, 0.1], [2.0, 0.0, 1.0], 1.0, 10, 0.85, int(seed[0]))
    want = np.zeros((3, 3))
    for w, l, wt in d["yeti_gt_competitors"]:
        want[int(w), int(l)] = wt
    assert np.max(np.abs(got - want)) <= TOL  # the log prints 6 decimals
    assert np.count_nonzero(got) == len(d["yeti_gt_competitors"])


def test_yetirank_tree_seeder_matches_trainer_log():
    # update_pairs events per tree: the derivative, leaf-value and learning-fold
    # recalc seeds (the seeder draws the learning fold's before the leaf values')
    d = _load()
    gt = d["yeti_gt_recalc_seeds"]
    ours = oracle.yeti_recalc_seeds(20260617, 5, 4, 2, gt.shape[0])
    np.testing.assert_array_equal(ours[:, [0, 2, 1]], gt)


def test_stochasticrank_noise_matches_trainer_log():
    # each logged draw: seed = recalc base + group index, one std_normal per
    # document per sample, in document order
    d = _load()
    seeds, rows = d["srank_gt_noise_seed"], d["srank_gt_noise"]
    streams = {}
    for s, (sample, doc, count, noise) in zip(seeds, rows):
        key = int(s)
        if key not in streams:
            streams[key] = oracle.TFastRng64(key)
        assert int(doc) < int(count)
        got = streams[key].std_normal()
        assert abs(got - noise) <= 1e-12
    # every logged stream is a derivative or leaf-value recalc base of the
    # corpus fit (random_seed 20260617, 5 groups, 4 features, depth 2) + group
    bases = oracle.yeti_recalc_seeds(20260617, 5, 4, 2, 5)[:, [0, 2]].ravel()
    valid = {(int(b) + g) % 2**64 for b in bases for g in range(5)}
    assert {int(s) for s in seeds} <= valid


def test_lambdamart_no_op_metrics_leave_zero_ders():
    # MRR / ERR / MAP: the reference accepts the metric and leaves every der at
    # zero (crates/cb-compute/src/ranking_der.rs:574-581), so the leaves are 0
    rs = np.random.RandomState(4)
    offsets = np.array([0, 7, 15, 30, 41], dtype=np.int64)
    n = int(offsets[-1])
    bins = rs.randint(0, 9, size=(3, n)).astype(np.uint8)
    y = rs.randint(0, 4, size=n).astype(np.float64)
    kw = dict(loss="LambdaMart", depth=2, iterations=2, learning_rate=0.3, l2_leaf_reg=1.0)
    base = oracle.train_ranking(bins, [8, 8, 8], y, offsets, **kw)
    assert np.any(base.raw_leaf_values)  # NDCG trains
    for metric in ("MRR", "ERR", "MAP"):
        o = oracle.train_ranking(bins, [8, 8, 8], y, offsets, lambdamart_metric=metric, **kw)
        assert not np.any(o.raw_leaf_values) and not np.any(o.staged)


def test_pairlogit_pair_weight_scales_ders():
    # the reference's vector (crates/cb-compute/src/ranking_der_test.rs:314):
    # approx [0, 0], document 0 beats document 1 with weight w: der1 = [w/2,
    # -w/2], der2 = [-w/4, -w/4].  A depth-1 tree splits the two documents
    # apart, so each raw Newton leaf is der1 / (-der2 + c) for the same l2
    # term c: w/2 / (w/4 + c) for the winner's leaf.
    bins = np.array([[1, 0]], dtype=np.uint8)
    y = np.array([1.0, 0.0])
    offsets = np.array([0, 2], dtype=np.int64)
    pairs = np.array([[0, 1]], dtype=np.int64)
    kw = dict(loss="PairLogit", pairs=pairs, depth=1, iterations=1, learning_rate=0.1, l2_leaf_reg=1.0)
    r1 = oracle.train_ranking(bins, [1], y, offsets, **kw).raw_leaf_values[0]
    r2 = oracle.train_ranking(bins, [1], y, offsets, pair_weights=[2.0], **kw).raw_leaf_values[0]
    c = 0.5 / r1[1] - 0.25  # from the unit-weight fit
    assert c > 0
    assert np.isclose(r1[0], -r1[1]) and np.isclose(r2[0], -r2[1])
    assert np.isclose(r2[1], 1.0 / (0.5 + c), rtol=1e-12)
