"""The CatBoost JSON model format for the oblivious models this package trains.

The reference reads and writes this format in crates/cb-model/src/json.rs
(save_json / load_json, :536-736 and :736-910).  It is upstream CatBoost's
`model.json` layout:

- `features_info.float_features[f]`: the feature's borders (NaN sentinels
  included: -f32::MAX first under nan_mode Min, f32::MAX last under Max),
  `has_nans`, and `nan_value_treatment` (AsIs / AsFalse / AsTrue).
- `oblivious_trees[t].splits[l]`: the split of level l, with `border`,
  `float_feature_index`, `split_index` (the border's index in the
  concatenation of all features' border lists) and
  `split_type = "FloatFeature"`.
- `oblivious_trees[t].leaf_values`: LEAF-major, `leaf * dim + d`.
  `oblivious_trees[t].leaf_weights`: one per leaf.
- `scale_and_bias`: `[1, [bias_d ...]]`.
- `model_info.class_params.class_to_label` for multi-dimensional models.

One-hot and CTR splits are not representable here, as in the reference
(json.rs:536-543).  Models carrying them raise ValueError.
"""
from __future__ import annotations

import json
from typing import Union

import numpy as np

from .boosting import MultiClassModel, ObliviousModel

_FLT_MAX = float(np.finfo(np.float32).max)


def _nan_fields(borders) -> tuple:
    b = list(borders)
    if b and b[0] == -_FLT_MAX:
        return True, "AsFalse"
    if b and b[-1] == _FLT_MAX:
        return True, "AsTrue"
    return False, "AsIs"


def to_json(model: Union[ObliviousModel, MultiClassModel]) -> dict:
    """The model as a CatBoost model.json document."""
    borders = [np.asarray(b, dtype=np.float64) for b in model.borders]
    F = len(borders)
    if getattr(model, "cat_values", None) or (np.asarray(model.split_feature) >= F).any():
        raise ValueError("one-hot splits cannot be represented in model.json; the reference saves them as .cbm")
    lv = np.asarray(model.leaf_values, dtype=np.float64)
    T, D = np.asarray(model.split_feature).shape
    L = 1 << D
    dim = 1 if lv.ndim == 2 else lv.shape[2]
    offset = np.concatenate([[0], np.cumsum([len(b) for b in borders])]).astype(np.int64)
    weights = getattr(model, "leaf_weights", None)
    floats = []
    for f, b in enumerate(borders):
        has_nans, treatment = _nan_fields(b)
        floats.append({"borders": [float(v) for v in b], "feature_id": "", "feature_index": f,
                       "flat_feature_index": f, "has_nans": has_nans, "nan_value_treatment": treatment})
    trees = []
    for t in range(T):
        splits = []
        for l in range(D):
            f, b = int(model.split_feature[t, l]), int(model.split_bin[t, l])
            splits.append({"border": float(borders[f][b]), "float_feature_index": f,
                           "split_index": int(offset[f] + b), "split_type": "FloatFeature"})
        leaf = lv[t].reshape(L, dim)  # leaf-major on the wire
        lw = np.zeros(L) if weights is None else np.asarray(weights[t], dtype=np.float64)
        trees.append({"leaf_values": [float(v) for v in leaf.reshape(-1)], "leaf_weights": [float(v) for v in lw],
                      "splits": splits})
    bias = float(getattr(model, "bias", 0.0) or 0.0)
    doc = {"features_info": {"float_features": floats}, "oblivious_trees": trees,
           "scale_and_bias": [1, [bias] * dim]}
    if dim > 1:
        doc["model_info"] = {"class_params": {"class_to_label": list(range(dim))}}
    return doc


def save_json(model: Union[ObliviousModel, MultiClassModel], path: str) -> None:
    with open(path, "w") as fh:
        json.dump(to_json(model), fh)


def from_json(doc: Union[dict, str]) -> Union[ObliviousModel, MultiClassModel]:
    """A model.json document (dict or JSON text) as an ObliviousModel (one
    output dimension) or a MultiClassModel; leaf weights ride along in
    `leaf_weights`."""
    if isinstance(doc, str):
        doc = json.loads(doc)
    floats = doc["features_info"].get("float_features", [])
    borders = [np.asarray(f.get("borders") or [], dtype=np.float64) for f in floats]
    sb = doc.get("scale_and_bias", [1, [0.0]])
    scale, bias = float(sb[0]), [float(v) for v in sb[1]]
    if scale != 1.0:
        raise ValueError(f"scale {scale} is not supported")
    dim = max(1, len(bias))
    trees = doc.get("oblivious_trees", [])
    if not trees:
        raise ValueError("no oblivious trees")
    D = len(trees[0]["splits"])
    L = 1 << D
    T = len(trees)
    sf = np.zeros((T, D), dtype=np.int32)
    sbin = np.zeros((T, D), dtype=np.int32)
    lv = np.zeros((T, L, dim), dtype=np.float64)
    lw = np.zeros((T, L), dtype=np.float64)
    for t, tree in enumerate(trees):
        if len(tree["splits"]) != D:
            raise ValueError("trees of different depths")
        for l, s in enumerate(tree["splits"]):
            if s.get("split_type", "FloatFeature") != "FloatFeature":
                raise ValueError(f"split type {s.get('split_type')} is not supported")
            f = int(s["float_feature_index"])
            hit = np.flatnonzero(borders[f] == float(s["border"]))
            if hit.size != 1:
                raise ValueError(f"border {s['border']} is not in feature {f}'s border list")
            sf[t, l], sbin[t, l] = f, int(hit[0])
        vals = np.asarray(tree["leaf_values"], dtype=np.float64)
        if vals.size != L * dim:
            raise ValueError(f"tree {t}: {vals.size} leaf values, expected {L * dim}")
        lv[t] = vals.reshape(L, dim)
        w = tree.get("leaf_weights") or []
        if len(w) == L:
            lw[t] = w
    if dim == 1:
        m = ObliviousModel(borders, sf, sbin, lv[:, :, 0], bias[0])
    else:
        if any(b != 0.0 for b in bias):
            raise ValueError("a multi-dimensional bias is not supported")
        m = MultiClassModel(borders, sf, sbin, lv)
    m.leaf_weights = lw
    return m


def load_json(path: str) -> Union[ObliviousModel, MultiClassModel]:
    with open(path) as fh:
        return from_json(json.load(fh))

