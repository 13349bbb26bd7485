"""The CatBoost binary model file (.cbm) reader / writer against upstream files.

tests/golden/model_cbm.npz holds seven upstream CatBoost 1.2.10 .cbm files
from the reference's fixtures (the format of crates/cb-model/src/cbm.rs),
with the same models' model.json where upstream wrote one and upstream's
predictions for model_sum.  Checked here:

- every file decodes (FlatBuffers offsets, counts and alignment verified),
  and where a model.json exists the decoded model equals the JSON one field
  for field (borders, splits, leaf values, bias);
- the model_sum models predict upstream's values through the oracle's apply
  (crates/cb-model/src/apply.rs:374-410);
- the one-hot fits' decoded splits and leaves equal upstream's (float splits
  by border, one-hot splits by category hash);
- writing a decoded model and reading it back gives the same model and the
  same core fields (TreeSplits, borders, leaves, bias); writing is
  deterministic;
- this package's own models round-trip, one-hot categories are written as
  CalcCatFeatureHash (checked against the reference's hash vectors and the
  oracle's CityHash64), and the one-hot fit that the oracle trains on
  upstream's rows writes the same (feature, category hash) splits as
  upstream's own file;
- malformed files raise ValueError.
"""
import json
import os
import random
import struct

import numpy as np
import pytest

from oracle import oracle

from catboost_rs_b200 import MultiClassModel, ObliviousModel, model_cbm, model_json
from catboost_rs_b200.cat_hash import cat_feature_hash, city_hash64

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "model_cbm.npz")
ONE_HOT = os.path.join(HERE, "golden", "one_hot.npz")
FMAX = float(np.finfo(np.float32).max)
FILES = ["model_sum_m0", "model_sum_m1", "mae", "partial_dependence", "staged_predict", "one_hot_default_binary",
         "one_hot_multi"]


def _z():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def _bytes(name):
    return _z()[name + "__cbm"].tobytes()


def _same_model(a, b):
    np.testing.assert_array_equal(a.split_feature, b.split_feature)
    np.testing.assert_array_equal(a.split_bin, b.split_bin)
    np.testing.assert_array_equal(a.leaf_values, b.leaf_values)
    assert len(a.borders) == len(b.borders)
    for x, y in zip(a.borders, b.borders):
        np.testing.assert_array_equal(x, y)
    assert getattr(a, "bias", 0.0) == getattr(b, "bias", 0.0)
    ca, cb_ = getattr(a, "cat_values", None), getattr(b, "cat_values", None)
    assert (ca is None) == (cb_ is None)
    if ca is not None:
        assert [list(map(int, c)) for c in ca] == [list(map(int, c)) for c in cb_]


@pytest.mark.parametrize("name", FILES)
def test_upstream_file_decodes(name):
    core = model_cbm.read_core(_bytes(name))
    assert core["FormatVersion"] == "FlabuffersModel_v1"
    t = core["ModelTrees"]
    assert len(t["TreeSizes"]) == len(t["TreeStartOffsets"]) > 0
    m = model_cbm.from_core(core)
    T, D = m.split_feature.shape
    assert m.leaf_values.shape[:2] == (T, 1 << D)


@pytest.mark.parametrize("name", ["mae", "partial_dependence"])
def test_decoded_equals_upstream_model_json(name):
    z = _z()
    _same_model(model_cbm.from_cbm_bytes(_bytes(name)), model_json.from_json(str(z[name + "__json"])))


@pytest.mark.parametrize("m", ["m0", "m1"])
def test_model_sum_predicts_as_upstream(m):
    z = _z()
    model = model_cbm.from_cbm_bytes(_bytes("model_sum_" + m))
    X = z["model_sum__X"]
    flat = oracle.flatten_oblivious(model.split_feature, model.split_borders(), model.leaf_values)
    nan_above = np.array([len(b) > 0 and b[-1] == FMAX for b in model.borders], dtype=np.uint8)
    got = oracle.apply_oblivious(np.ascontiguousarray(X.T, dtype=np.float32), flat, model.bias, nan_above)
    assert np.max(np.abs(got - z["model_sum__expected_" + m])) <= 1e-9


def _onehot():
    z = np.load(ONE_HOT)
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("sc", ["default_binary", "multi"])
def test_one_hot_file_matches_upstream_fit(sc):
    d = _onehot()
    m = model_cbm.from_cbm_bytes(_bytes("one_hot_" + sc))
    F = len(m.borders)
    assert F == json.loads(str(d[f"{sc}__params"]))["n_float"]
    kind, feat, val = d[f"{sc}__split_kind"], d[f"{sc}__split_feature"], d[f"{sc}__split_value"]
    T, D = kind.shape
    for t in range(T):
        for l in range(D):
            f, b = int(m.split_feature[t, l]), int(m.split_bin[t, l])
            if kind[t, l] == 0:
                assert f == feat[t, l] and np.float32(m.borders[f][b]) == np.float32(val[t, l])
            else:
                assert f - F == feat[t, l] and (int(m.cat_values[f - F][b]) & 0xFFFFFFFF) == int(val[t, l])
    np.testing.assert_array_equal(m.leaf_values[:, :, 0], d[f"{sc}__leaf_values"])


@pytest.mark.parametrize("name", FILES)
def test_write_read_round_trip(name):
    up = model_cbm.read_core(_bytes(name))
    m = model_cbm.from_core(up)
    data = model_cbm.to_cbm_bytes(m)
    assert data == model_cbm.to_cbm_bytes(m)  # deterministic
    ours = model_cbm.read_core(data)
    _same_model(m, model_cbm.from_core(ours))
    a, b = up["ModelTrees"], ours["ModelTrees"]
    for k in ("TreeSplits", "TreeSizes", "TreeStartOffsets", "LeafValues"):
        np.testing.assert_array_equal(a[k], b[k])
    assert a["ApproxDimension"] == b["ApproxDimension"]
    up_bias = a["MultiBias"] if len(a.get("MultiBias", [])) else [a["Bias"]]
    np.testing.assert_array_equal(np.asarray(up_bias), b["MultiBias"])
    for fa, fb in zip(a["FloatFeatures"], b["FloatFeatures"]):
        np.testing.assert_array_equal(fa["Borders"], fb["Borders"])
        assert (fa["HasNans"], fa["Index"], fa["NanValueTreatment"]) == (fb["HasNans"], fb["Index"],
                                                                         fb["NanValueTreatment"])
    assert [(o["Index"], list(o["Values"])) for o in a["OneHotFeatures"]] == \
        [(o["Index"], list(o["Values"])) for o in b["OneHotFeatures"]]


def test_trained_model_round_trip(tmp_path):
    rs = np.random.RandomState(0)
    borders = [np.sort(rs.standard_normal(5).astype(np.float32)).astype(np.float64), np.array([-FMAX, 0.0, 1.0]),
               np.array([0.5, FMAX])]
    sf = rs.randint(0, 3, (4, 3)).astype(np.int32)
    sb = np.array([[rs.randint(len(borders[f])) for f in row] for row in sf], dtype=np.int32)
    m = ObliviousModel(borders, sf, sb, rs.standard_normal((4, 8)), 0.25)
    path = os.path.join(tmp_path, "m.cbm")
    model_cbm.save_cbm(m, path, info={"note": "test"})
    r = model_cbm.load_cbm(path)
    _same_model(m, r)
    assert r.info == {"note": "test"}
    core = model_cbm.read_core(open(path, "rb").read())
    assert [f["NanValueTreatment"] for f in core["ModelTrees"]["FloatFeatures"]] == ["AsIs", "AsFalse", "AsTrue"]
    # the same model through model.json agrees
    _same_model(model_json.from_json(model_json.to_json(m)), r)


def test_multiclass_and_one_hot_round_trip():
    rs = np.random.RandomState(1)
    borders = [np.array([-1.0, 0.0, 2.5]), np.array([0.25])]
    cats = [["red", "green", "blue"], ["x", "y"]]
    sf = np.array([[0, 2, 3], [1, 2, 0]], dtype=np.int32)
    sb = np.array([[1, 2, 1], [0, 0, 2]], dtype=np.int32)
    m = MultiClassModel(borders, sf, sb, rs.standard_normal((2, 8, 3)), cat_values=cats)
    data = model_cbm.to_cbm_bytes(m)
    core = model_cbm.read_core(data)
    assert core["ModelTrees"]["ApproxDimension"] == 3
    assert json.loads(core["InfoMap"]["class_params"])["class_to_label"] == [0, 1, 2]
    r = model_cbm.from_cbm_bytes(data)
    assert r.cat_values_are_hashes
    assert [[int(v) & 0xFFFFFFFF for v in c] for c in r.cat_values] == \
        [[oracle.cat_hash(s) for s in c] for c in cats]
    np.testing.assert_array_equal(r.split_feature, sf)
    np.testing.assert_array_equal(r.split_bin, sb)
    np.testing.assert_array_equal(r.leaf_values, m.leaf_values)
    # rewriting a loaded model keeps its hashes as they are
    assert model_cbm.to_cbm_bytes(r) == data


def test_oracle_one_hot_fit_writes_upstream_splits():
    """Train the one_hot_train/multi fit with the oracle on upstream's rows,
    write it with this package's writer, and compare the written (feature,
    category hash) splits and the leaves with upstream's own .cbm file (a level
    where a binary column's complementary test was chosen is compared with its
    leaf bit flipped, as the oracle's one-hot test documents)."""
    d = _onehot()
    sc = "multi"
    p = json.loads(str(d[f"{sc}__params"]))
    X = d[f"{sc}__X"]
    cat_cols = d[f"{sc}__cat"]
    F = p["n_float"]
    borders = [d[f"{sc}__borders{f}"] for f in range(F)]
    bins = oracle.quantize(np.ascontiguousarray(X.T), borders)
    seen, cat_bins = [], []
    for col in cat_cols:
        b, s = oracle.perfect_hash_bins([str(v) for v in col])
        cat_bins.append(b)
        seen.append(s)
    fit = oracle.train(bins, [len(b) for b in borders], d[f"{sc}__y"], loss=p["loss"], depth=p["depth"],
                       iterations=p["iterations"], learning_rate=p["learning_rate"], l2_leaf_reg=p["l2_leaf_reg"],
                       score_function=p["score_function"], bootstrap_type="No", boost_from_average=False,
                       staged=True, cat_bins_fm=np.array(cat_bins))
    ours = MultiClassModel(borders, fit.split_feature, fit.split_bin, fit.leaf_values[:, :, None], cat_values=seen)
    mine = model_cbm.from_cbm_bytes(model_cbm.to_cbm_bytes(ours))
    up = model_cbm.from_cbm_bytes(_bytes("one_hot_" + sc))
    T, D = up.split_feature.shape
    for t in range(T):
        flip = 0
        for l in range(D):
            fm, fu = int(mine.split_feature[t, l]), int(up.split_feature[t, l])
            assert fm == fu, (t, l)
            if fm < F:
                assert mine.borders[fm][mine.split_bin[t, l]] == up.borders[fu][up.split_bin[t, l]]
                continue
            hm = int(mine.cat_values[fm - F][mine.split_bin[t, l]]) & 0xFFFFFFFF
            hu = int(up.cat_values[fu - F][up.split_bin[t, l]]) & 0xFFFFFFFF
            if hm != hu:  # the complementary test of a binary column
                assert len(seen[fm - F]) == 2
                flip |= 1 << l
        lv = mine.leaf_values[t, :, 0][np.arange(1 << D) ^ flip]
        assert np.max(np.abs(lv - up.leaf_values[t, :, 0])) <= 1e-5, t


def test_cat_hash_matches_reference_vectors_and_oracle():
    d = _onehot()
    for s, h32, h64 in zip(d["hash_strings"], d["hash_ui32"], d["hash_ui64"]):
        assert city_hash64(str(s).encode()) == int(h64)
        assert cat_feature_hash(str(s)) == int(h32)
    rs = random.Random(7)
    for n in list(range(0, 130)) + [200, 255, 256, 257, 1000]:
        s = "".join(chr(rs.randrange(32, 127)) for _ in range(n))
        assert city_hash64(s.encode()) == oracle.city_hash64(s), n


def test_malformed_files_are_rejected():
    good = model_cbm.to_cbm_bytes(model_cbm.from_cbm_bytes(_bytes("mae")))
    cases = {
        "magic": b"CBM2" + good[4:],
        "short": good[:6],
        "size": good[:4] + struct.pack("<I", len(good)) + good[8:],
        "tail": good + b"\0" * 8,
        "root": good[:8] + struct.pack("<I", len(good) * 4) + good[12:],
        "truncated": good[:4] + struct.pack("<I", len(good) // 2 - 8) + good[8:len(good) // 2],
    }
    for name, data in cases.items():
        with pytest.raises(ValueError):
            model_cbm.from_cbm_bytes(data)
    # every single corrupted byte either still decodes to a model or raises ValueError
    rs = np.random.RandomState(3)
    for pos in rs.choice(np.arange(8, len(good)), size=200, replace=False):
        bad = bytearray(good)
        bad[pos] ^= 0xFF
        try:
            model_cbm.from_cbm_bytes(bytes(bad))
        except ValueError:
            pass


def test_unsupported_sections_are_rejected():
    core = model_cbm.read_core(_bytes("mae"))
    core["ModelTrees"]["HasCtrFeatures"] = True
    with pytest.raises(ValueError, match="CtrFeatures"):
        model_cbm.from_core(core)
    core = model_cbm.read_core(_bytes("mae"))
    core["FormatVersion"] = "FlatbuffersModel_v1"
    with pytest.raises(ValueError, match="FormatVersion"):
        model_cbm.from_core(core)


@pytest.mark.gpu
def test_device_fit_round_trips_through_cbm(tmp_path):
    """A model trained on the device, written to .cbm and read back, predicts
    bit-identically through the device apply."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    rs = np.random.RandomState(5)
    n, F = 20000, 8
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.rand(n, F) < 0.05] = np.nan
    y = (X[:, 0] > 0.3).astype(np.float64)
    borders = []
    for f in range(F):
        q = np.nanquantile(X[:, f].astype(np.float64), np.linspace(0, 1, 34)[1:-1])
        b = np.unique(q.astype(np.float32).astype(np.float64))
        borders.append(np.concatenate([[-FMAX], b]))  # nan_mode Min sentinel
    fp = cb.FitParams(loss="Logloss", depth=6, iterations=20, learning_rate=0.1, l2_leaf_reg=3.0,
                      score_function="Cosine", bootstrap_type="Bayesian", boost_from_average=False)
    m = cb.fit([np.ascontiguousarray(X[:, f]) for f in range(F)], borders, y, fp, staged=False)
    path = os.path.join(tmp_path, "fit.cbm")
    cb.save_cbm(m, path)
    r = cb.load_cbm(path)
    _same_model(m, r)
    np.testing.assert_array_equal(r.predict(X), m.predict(X))
