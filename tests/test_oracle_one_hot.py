"""Pin the oracle's one-hot categorical features to upstream.

tests/golden/one_hot.npz holds the reference's CityHash vectors
(crates/cb-oracle/fixtures/cat_hash: CalcCatFeatureHash = the low 32 bits of
CityHash64 of the category's string form, crates/cb-data/src/cat_hash.rs, and
the first-seen perfect-hash bins) and two upstream CatBoost 1.2.10 Logloss fits
with one-hot categorical features (crates/cb-oracle/fixtures/one_hot_train).
A one-hot candidate is an equality split on one perfect-hash bin, scored with
TRUE = the bin's cell and FALSE = the parent total minus it
(histogram.rs:1160-1290), one candidate per distinct learn-set bin ascending,
after every float candidate (tree.rs:1290-1380, 3606-3615).

On a binary categorical column the two equality tests induce the same
partition with the children swapped, so their scores tie exactly; first-wins
over the first-seen bins picks bin 0 where upstream sometimes picks the other
value.  The comparison therefore maps such a level onto upstream's by
flipping that leaf bit (the reference's own one_hot_oracle_test.rs:240-345
documents the same).  The reference leaves its `multi` comparison ignored
(one_hot_oracle_test.rs:240-350 records a tree-2 divergence on a
cardinality-3 column); this restatement matches upstream on all three trees
of both fits.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "one_hot.npz")
TOL = 1e-5


def _load():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def test_cat_hash_vectors():
    d = _load()
    for s, h32, h64 in zip(d["hash_strings"], d["hash_ui32"], d["hash_ui64"]):
        assert oracle.city_hash64(str(s)) == int(h64), s
        assert oracle.cat_hash(str(s)) == int(h32), s


def test_perfect_hash_bins_first_seen():
    d = _load()
    n = d["hash_bins"].size // 2
    order = {0: [str(v) for v in d["hash_c0_order"]], 1: [str(v) for v in d["hash_c1_order"]]}
    h = d["hash_per_object"]
    for c in (0, 1):
        labels = {oracle.cat_hash(s): s for s in order[c]}
        col = [labels[int(v)] for v in h[c * n:(c + 1) * n]]
        bins, seen = oracle.perfect_hash_bins(col)
        np.testing.assert_array_equal(bins, d["hash_bins"][c * n:(c + 1) * n])
        assert seen == order[c]


def _fit(d, sc):
    p = json.loads(str(d[f"{sc}__params"]))
    X = d[f"{sc}__X"]
    F = p["n_float"]
    borders = [d[f"{sc}__borders{f}"] for f in range(F)]
    bins = oracle.quantize(X.T.copy(), borders)
    cats = d[f"{sc}__cat"]
    cat_bins, seen = [], []
    for col in cats:
        b, s = oracle.perfect_hash_bins([str(v) for v in col])
        cat_bins.append(b)
        seen.append(s)
    assert p["leaf_estimation_method"] == "Gradient"
    fit = oracle.train(bins, [len(b) for b in borders], d[f"{sc}__y"], loss=p["loss"], depth=p["depth"],
                       iterations=p["iterations"], learning_rate=p["learning_rate"], l2_leaf_reg=p["l2_leaf_reg"],
                       score_function=p["score_function"], boost_from_average=False, cat_bins_fm=np.array(cat_bins))
    return p, borders, seen, fit


@pytest.mark.parametrize("sc,trees", [("default_binary", 3), ("multi", 3)])
def test_one_hot_fit_matches_upstream(sc, trees):
    d = _load()
    p, borders, seen, fit = _fit(d, sc)
    F = p["n_float"]
    kind, feat, val = d[f"{sc}__split_kind"], d[f"{sc}__split_feature"], d[f"{sc}__split_value"]
    D = kind.shape[1]
    n_one_hot = 0
    for t in range(trees):
        flip = 0
        for l in range(D):
            f, b = int(fit.split_feature[t, l]), int(fit.split_bin[t, l])
            if kind[t, l] == 0:
                assert f == feat[t, l] and np.float32(borders[f][b]) == np.float32(val[t, l]), (t, l)
                continue
            n_one_hot += 1
            assert f - F == feat[t, l], (t, l)
            values = seen[f - F]
            h = oracle.cat_hash(values[b])
            if h != int(val[t, l]):
                # the complementary test of a binary column: the same partition
                assert len(values) == 2 and oracle.cat_hash(values[1 - b]) == int(val[t, l]), (t, l)
                flip |= 1 << l
        ours = fit.leaf_values[t][np.arange(1 << D) ^ flip]
        assert np.max(np.abs(ours - d[f"{sc}__leaf_values"][t])) <= TOL, t
    assert n_one_hot > 0  # the fixture exercises one-hot splits
    if trees == kind.shape[0]:
        assert np.max(np.abs(fit.final_approx - d[f"{sc}__predictions"])) <= TOL


def test_one_hot_rejected_with_draws():
    # upstream rejects one-hot columns whenever draws are active (bootstrap or
    # random strength): the perturbed search has no established one-hot draw
    # accounting (tree.rs:1403-1420)
    d = _load()
    sc = "multi"
    X = d[f"{sc}__X"]
    borders = [d[f"{sc}__borders0"]]
    bins = oracle.quantize(X.T.copy(), borders)
    cat = np.array([oracle.perfect_hash_bins([str(v) for v in col])[0] for col in d[f"{sc}__cat"]])
    with pytest.raises(RuntimeError):
        oracle.train(bins, [1], d[f"{sc}__y"], loss="Logloss", depth=2, iterations=1, bootstrap_type="Bernoulli",
                     cat_bins_fm=cat)


def test_multiclass_one_hot_binary_column_equals_float_encoding():
    # on a two-category column the equality candidates {== bin 0, == bin 1}
    # induce the partitions of the float border between the bins, children
    # swapped for == 0: the same trees up to that leaf bit, the same fit
    rs = np.random.RandomState(4)
    n, K = 3000, 3
    X = rs.standard_normal((n, 2)).astype(np.float32)
    c = rs.randint(0, 2, n)
    cls = np.argmax(np.c_[X, c] @ rs.standard_normal((3, K)) + rs.gumbel(size=(n, K)), axis=1).astype(np.int32)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(2)]
    bins = oracle.quantize(X.T.copy(), borders)
    cat_bins, seen = oracle.perfect_hash_bins(list(c))
    as_float = np.vstack([bins, cat_bins.astype(np.uint8)])
    a = oracle.train_multiclass(bins, [len(b) for b in borders], cls, K, depth=3, iterations=3,
                                cat_bins_fm=cat_bins[None, :])
    b = oracle.train_multiclass(as_float, [len(b) for b in borders] + [1], cls, K, depth=3, iterations=3)
    assert (a.split_feature == 2).any()
    np.testing.assert_array_equal(a.split_feature, b.split_feature)
    np.testing.assert_allclose(a.final_approx, b.final_approx, rtol=0, atol=1e-12)
