"""Loading helpers for the committed golden fixtures (tests/golden/*.npz)."""
from __future__ import annotations

import glob
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def scenario_names():
    return sorted(os.path.basename(p)[4:-4] for p in glob.glob(os.path.join(GOLDEN, "e2e_*.npz")))


def load_scenario(name):
    z = np.load(os.path.join(GOLDEN, f"e2e_{name}.npz"), allow_pickle=False)
    d = {k: z[k] for k in z.files}
    d["params"] = json.loads(str(d["params"]))
    counts = d["border_counts"]
    offs = np.concatenate([[0], np.cumsum(counts)])
    d["borders"] = [d["borders_flat"][offs[i]:offs[i + 1]] for i in range(len(counts))]
    d["name"] = name
    return d


def scalar_vectors():
    with open(os.path.join(GOLDEN, "scalar_vectors.json")) as f:
        return json.load(f)


def apply_trees(X, borders, split_feature, split_bin, leaf_values, bias=0.0):
    """Oblivious-ensemble apply from quantized splits (float value > border)."""
    X = np.asarray(X, dtype=np.float32)
    out = np.full(X.shape[0], bias, dtype=np.float64)
    for t in range(split_feature.shape[0]):
        leaf = np.zeros(X.shape[0], dtype=np.int64)
        for l in range(split_feature.shape[1]):
            f = split_feature[t, l]
            if f < 0:
                continue
            b = borders[f][split_bin[t, l]]
            v = X[:, f].astype(np.float64)
            nan_max = len(borders[f]) > 0 and borders[f][-1] == np.float64(np.finfo(np.float32).max)
            # nan_mode=Max routes NaN above every border (histogram.rs bin_of)
            passes = (np.isnan(v) & nan_max) | (v > b)
            leaf |= passes.astype(np.int64) << l
        out += leaf_values[t][leaf]
    return out
