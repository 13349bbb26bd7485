"""The CatBoost model.json reader / writer against upstream documents.

tests/golden/model_json.npz holds five upstream CatBoost 1.2.10 model.json
documents from the reference's fixtures (the format of
crates/cb-model/src/json.rs).  Each is read into this package's model, applied
by the oracle's apply (crates/cb-model/src/apply.rs:374-410) against
upstream's predictions at the 1e-5 bar, and written back: the written
document must equal upstream's on every field the format carries (borders and
NaN treatment, splits with their split_index, leaf values and weights,
scale_and_bias).
"""
import json
import os

import numpy as np
import pytest

from golden_io import load_scenario
from oracle import oracle

from catboost_rs_b200 import model_json

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "model_json.npz")
TOL = 1e-5
FMAX = float(np.finfo(np.float32).max)
DOCS = ["regression_skeleton", "binclf_skeleton", "nan_mode_Max", "nan_mode_Min", "multiclass_softmax"]


def _doc(name):
    return json.loads(str(np.load(GOLDEN)[name]))


@pytest.mark.parametrize("name", DOCS)
def test_round_trip_equals_upstream(name):
    up = _doc(name)
    ours = model_json.to_json(model_json.from_json(up))
    uf, of = up["features_info"]["float_features"], ours["features_info"]["float_features"]
    assert len(uf) == len(of)
    for a, b in zip(uf, of):
        for k in ("borders", "feature_index", "flat_feature_index", "has_nans", "nan_value_treatment"):
            assert a[k] == b[k], (name, k)
    assert len(up["oblivious_trees"]) == len(ours["oblivious_trees"])
    for a, b in zip(up["oblivious_trees"], ours["oblivious_trees"]):
        assert a["splits"] == b["splits"]
        assert a["leaf_values"] == b["leaf_values"]
        assert a["leaf_weights"] == b["leaf_weights"]
    assert up["scale_and_bias"] == ours["scale_and_bias"]


@pytest.mark.parametrize("name,scenario,eval_key", [("regression_skeleton", "regression_skeleton", None),
                                                    ("binclf_skeleton", "binclf_skeleton", None),
                                                    ("nan_mode_Max", "nan_mode_Max", "eval"),
                                                    ("nan_mode_Min", "nan_mode_Min", "eval")])
def test_loaded_model_predicts_as_upstream(name, scenario, eval_key):
    m = model_json.from_json(_doc(name))
    sc = load_scenario(scenario)
    X, want = (sc["X_eval"], sc["preds_eval"]) if eval_key else (sc["X"], sc["staged"][-1])
    flat = oracle.flatten_oblivious(m.split_feature, m.split_borders(), m.leaf_values)
    nan_above = np.array([len(b) > 0 and b[-1] == FMAX for b in m.borders], dtype=np.uint8)
    got = oracle.apply_oblivious(np.ascontiguousarray(X.T, dtype=np.float32), flat, m.bias, nan_above)
    assert np.max(np.abs(got - want)) <= TOL


def test_multiclass_document_layout():
    up = _doc("multiclass_softmax")
    m = model_json.from_json(up)
    K = len(up["scale_and_bias"][1])
    assert m.leaf_values.shape[2] == K  # leaf-major on the wire, [T, L, K] in memory
    tree0 = up["oblivious_trees"][0]["leaf_values"]
    np.testing.assert_array_equal(m.leaf_values[0].reshape(-1), tree0)
    assert model_json.to_json(m)["model_info"]["class_params"]["class_to_label"] == list(range(K))


def test_trained_model_round_trip(tmp_path):
    rs = np.random.RandomState(0)
    borders = [np.sort(rs.standard_normal(5)), np.array([-FMAX, 0.0, 1.0]), np.array([0.5, FMAX])]
    sf = rs.randint(0, 3, (4, 3)).astype(np.int32)
    sb = np.array([[rs.randint(len(borders[f])) for f in row] for row in sf], dtype=np.int32)
    from catboost_rs_b200 import ObliviousModel
    m = ObliviousModel(borders, sf, sb, rs.standard_normal((4, 8)), 0.25)
    path = os.path.join(tmp_path, "m.json")
    model_json.save_json(m, path)
    r = model_json.load_json(path)
    np.testing.assert_array_equal(r.split_feature, sf)
    np.testing.assert_array_equal(r.split_bin, sb)
    np.testing.assert_array_equal(r.leaf_values, m.leaf_values)
    assert r.bias == 0.25
    d = model_json.to_json(m)
    assert [f["nan_value_treatment"] for f in d["features_info"]["float_features"]] == ["AsIs", "AsFalse", "AsTrue"]


def test_one_hot_models_are_rejected():
    from catboost_rs_b200 import MultiClassModel
    m = MultiClassModel([np.array([0.0])], np.array([[1]], dtype=np.int32), np.array([[0]], dtype=np.int32),
                        np.zeros((1, 2, 3)), cat_values=[["a", "b"]])
    with pytest.raises(ValueError, match="one-hot"):
        model_json.to_json(m)
