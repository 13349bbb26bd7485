"""Regenerate the golden fixtures in this directory from the reference checkout.

Run once, in the build container where the reference is mounted:

    python tests/golden/make_golden.py /path/to/catboost_rs

It reads only the reference's committed TEST data -- the golden vectors that
its unit tests pin (TFastRng64 / std_normal values transcribed from upstream
fast_ut.cpp, the FastLogf bit-pattern table) and the upstream CatBoost 1.2.10
end-to-end fixtures its oracle tests train against -- and writes them as small
.json / .npz files, so the GPU box (which has no reference checkout) can run
the same parity checks.  No reference source code is copied.
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np

OUT = os.path.dirname(os.path.abspath(__file__))


def _read(path):
    with open(path) as f:
        return f.read()


def scalar_vectors(ref):
    """Known-answer vectors from crates/cb-core/src/{rng,normal}_test.rs."""
    rng_t = _read(os.path.join(ref, "crates/cb-core/src/rng_test.rs"))
    first = int(re.search(r"rng\.gen_rand\(\),\s*([0-9_]+)_u64", rng_t).group(1).replace("_", ""))
    seq = re.search(r"EXPECTED: \[u64; 20\] = \[(.*?)\];", rng_t, re.S).group(1)
    uniform = [int(x) for x in re.findall(r"\d+", seq)]
    norm_t = _read(os.path.join(ref, "crates/cb-core/src/normal_test.rs"))
    vals = re.findall(r"\(n(\w*)\s*-\s*\(?(-?[0-9_.]+e-?\d+)\)?\)\.abs\(\)", norm_t)
    normals = {}
    for name, v in vals:
        normals.setdefault(name, float(v.replace("_", "")))
    red_t = _read(os.path.join(ref, "crates/cb-core/src/reduction_test.rs"))
    has_order_lock = "1e16" in red_t
    fx = os.path.join(ref, "crates/cb-train/tests/fixtures/fast_approx_ref.txt")
    logf = []
    for line in _read(fx).splitlines():
        p = line.split()
        if len(p) == 3 and p[0] == "fast_logf":
            logf.append([int(p[1], 16), int(p[2], 16)])
    return {
        "source": "crates/cb-core/src/rng_test.rs, normal_test.rs, reduction_test.rs; "
                  "crates/cb-train/tests/fixtures/fast_approx_ref.txt",
        "from_seed_17_first_gen_rand": first,
        "new_0_1_2_3_uniform_100": uniform,
        "std_normal": {
            "seed17_first": normals.get("1"),
            "seed17_second": normals.get("2"),
            "seed0_first": normals.get("0"),
            "seed42_first": normals.get("42"),
            "seed17_draws": [4, 2],
        },
        "sum_f64_order_lock": {"values": [1e16, 1.0, -1e16], "expected": 0.0,
                               "present_in_reference": has_order_lock},
        "fast_logf_bits": logf,
    }


def _tree_arrays(model, borders):
    trees = model["oblivious_trees"]
    depth = max(len(t["splits"]) for t in trees)
    T = len(trees)
    sf = np.full((T, depth), -1, dtype=np.int32)
    sv = np.full((T, depth), np.nan, dtype=np.float64)
    lv = np.zeros((T, 1 << depth), dtype=np.float64)
    for i, t in enumerate(trees):
        for l, s in enumerate(t["splits"]):
            sf[i, l] = s["float_feature_index"]
            sv[i, l] = s["border"]
        v = np.asarray(t["leaf_values"], dtype=np.float64)
        lv[i, : v.size] = v
    return sf, sv, lv


def _save(name, X, y, borders, params, model, staged=None, weights=None, extra=None):
    sf, sv, lv = _tree_arrays(model, borders)
    counts = np.array([len(b) for b in borders], dtype=np.int32)
    flat = np.concatenate([np.asarray(b, dtype=np.float64) for b in borders]) if counts.sum() else np.zeros(0)
    arrays = dict(X=np.asarray(X, dtype=np.float32), y=np.asarray(y, dtype=np.float64),
                  borders_flat=flat, border_counts=counts, split_feature=sf, split_border=sv,
                  leaf_values=lv, params=np.array(json.dumps(params)))
    if staged is not None:
        arrays["staged"] = np.asarray(staged, dtype=np.float64).reshape(lv.shape[0], -1)
    if weights is not None:
        arrays["weights"] = np.asarray(weights, dtype=np.float64)
    for k, v in (extra or {}).items():
        arrays[k] = v
    np.savez_compressed(os.path.join(OUT, f"e2e_{name}.npz"), **arrays)


def _params(cfg_params, loss):
    p = cfg_params
    return {
        "loss": loss,
        "depth": int(p["depth"]),
        "iterations": int(p["iterations"]),
        "learning_rate": float(p["learning_rate"]),
        "l2_leaf_reg": float(p["l2_leaf_reg"]),
        "score_function": p.get("score_function", "Cosine"),
        "bootstrap_type": p.get("bootstrap_type", "No").replace("MVS", "MVS"),
        "subsample": float(p.get("subsample", 0.66 if p.get("bootstrap_type") == "Bernoulli" else 0.8)),
        "bagging_temperature": float(p.get("bagging_temperature", 1.0)),
        "random_strength": float(p.get("random_strength", 0.0)),
        "random_seed": int(p.get("random_seed", 0)),
        "boost_from_average": bool(p.get("boost_from_average", False)),
    }


def e2e_fixtures(ref):
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    ld = lambda *p: np.load(os.path.join(fx, *p))  # noqa: E731
    jl = lambda *p: json.loads(_read(os.path.join(fx, *p)))  # noqa: E731
    written = []

    def borders_of(model):
        return [f["borders"] for f in model["features_info"]["float_features"]]

    # numeric_tiny skeletons (crates/cb-train/tests/slice_first_oracle_test.rs)
    Xt, yt = ld("inputs/numeric_tiny/X.npy"), ld("inputs/numeric_tiny/y.npy")
    for scen, loss in (("regression_skeleton", "RMSE"), ("binclf_skeleton", "Logloss")):
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        y = yt if loss == "RMSE" else (yt > np.median(yt)).astype(np.float64)
        _save(scen, Xt, y, borders_of(model), _params(cfg["params"], loss), model, ld(scen, "staged.npy"))
        written.append(scen)
    # regularization family on numeric_tiny
    for sub in ("l2", "bagging_temp", "random_strength", "random_strength_bernoulli"):
        scen = f"regularization/{sub}"
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        _save(scen.replace("/", "_"), Xt, yt, borders_of(model), _params(cfg["params"], "RMSE"), model,
              ld(scen, "staged.npy"))
        written.append(scen)
    # bootstrap families on the 1500-row multi-block input
    Xb, yb = ld("inputs/bootstrap_multiblock/X.npy"), ld("inputs/bootstrap_multiblock/y.npy")
    scen_list = [f"bootstrap/{k}" for k in ("no", "bayesian", "bernoulli", "mvs")]
    scen_list += [f"bootstrap_dev/{k}" for k in ("no", "bayesian", "bernoulli", "mvs")]
    scen_list += [f"mvs_seeds/s{s}_bfa{b}" for s in range(5) for b in (0, 1)]
    for scen in scen_list:
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        _save(scen.replace("/", "_"), Xb, yb, borders_of(model), _params(cfg["params"], "RMSE"), model,
              ld(scen, "staged.npy"))
        written.append(scen)
    # weighted / biased device-parity fixtures with their FULL border sets
    for scen in ("weighted_device_sym", "bias_device_sym"):
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        B = ld(scen, "borders.npy")
        w = ld(scen, "weights.npy") if os.path.exists(os.path.join(fx, scen, "weights.npy")) else None
        Xs = ld(scen, "X.npy")
        preds = ld(scen, "predictions.npy")
        _save(scen, Xs, ld(scen, "y.npy"), [list(r) for r in B], _params(cfg["params"], "RMSE"), model,
              weights=w, extra={"predictions": preds})
        written.append(scen)
    # Exact leaves: Quantile / MAE on numeric_tiny (model borders) and the
    # device-parity pair with their full frozen border sets
    for scen, alpha in (("quantile_alpha05_mae", 0.5), ("quantile_alpha07", 0.7)):
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        p = dict(_params(cfg["params"], "Quantile"), leaf_estimation_method="Exact", quantile_alpha=alpha,
                 quantile_delta=1e-6)
        _save(scen, Xt, yt, borders_of(model), p, model, ld(scen, "staged.npy"))
        written.append(scen)
    for sub, loss, alpha in (("mae", "MAE", 0.5), ("quantile07", "Quantile", 0.7)):
        scen = f"exact_leaf_device/{sub}"
        cfg, model = jl(scen, "config.json"), jl(scen, "model.json")
        p = dict(_params(cfg["params"], loss), leaf_estimation_method="Exact", quantile_alpha=alpha,
                 quantile_delta=1e-6)
        _save(f"exact_leaf_{sub}", ld(scen, "X.npy"), ld(scen, "y.npy"), [list(r) for r in ld(scen, "borders.npy")],
              p, model, extra={"predictions": ld(scen, "predictions.npy")})
        written.append(scen)
    # NaN handling, both sentinel modes (model borders carry the sentinel)
    cfg = jl("nan_mode", "config.json")
    for mode in ("Min", "Max"):
        model = jl("nan_mode", f"model_{mode}.json")
        _save(f"nan_mode_{mode}", ld("nan_mode", "X.npy"), ld("nan_mode", "y.npy"), borders_of(model),
              _params(cfg["params"], "RMSE"), model,
              extra={"X_eval": ld("nan_mode", "X_eval.npy").astype(np.float32),
                     "preds_eval": ld("nan_mode", f"preds_{mode}.npy")})
        written.append(f"nan_mode/{mode}")
    return written


def border_fixtures(ref):
    """Standalone upstream border sets (Pool.quantize().save_quantization_borders())
    from the reference's border_types/ and borders_quant/ fixtures, with the input
    columns narrowed to f32 (the reference narrows with `v as f32` before selecting)."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    inputs = {
        "borders_dense": "inputs/borders_dense/X.npy",
        "borders_runs": "inputs/borders_runs/X.npy",
        "numeric_nan": "inputs/numeric_nan/X.npy",
        "numeric_tiny": "inputs/numeric_tiny/X.npy",
        "float_only_byte_identity": "float_only_byte_identity/inputs/X.npy",
    }
    arrays = {f"X__{k}": np.load(os.path.join(fx, v)).astype(np.float32) for k, v in inputs.items()}
    cells = []
    cfg = json.loads(_read(os.path.join(fx, "border_types/config.json")))
    for stem, sc in sorted(cfg["scenarios"].items()):
        cells.append({"stem": stem, "dataset": sc["dataset"], "border_count": int(sc["border_count"]),
                      "border_type": sc["feature_border_type"], "nan_mode": sc["nan_mode"]})
        arrays[f"B__{stem}"] = np.load(os.path.join(fx, "border_types", f"{stem}.borders.npy"))
        arrays[f"C__{stem}"] = np.load(os.path.join(fx, "border_types", f"{stem}.borders_per_feature.npy"))
    qcfg = json.loads(_read(os.path.join(fx, "borders_quant/config.json")))
    for ds, sc in sorted(qcfg["scenarios"].items()):
        stem = f"quant.{ds}"
        cells.append({"stem": stem, "dataset": sc["input_dataset"], "border_count": int(sc["border_count"]),
                      "border_type": sc["border_selection_type"], "nan_mode": sc["nan_mode"]})
        arrays[f"B__{stem}"] = np.load(os.path.join(fx, "borders_quant", f"{ds}.borders.npy"))
        arrays[f"C__{stem}"] = np.load(os.path.join(fx, "borders_quant", f"{ds}.borders_per_feature.npy"))
    arrays["cells"] = np.array(json.dumps(cells))
    np.savez_compressed(os.path.join(OUT, "borders.npz"), **arrays)
    return [c["stem"] for c in cells]


def multiclass_fixture(ref):
    """Upstream MultiClass (softmax, Newton leaves) fixture on numeric_tiny:
    labels digitized at the 1/3 and 2/3 quantiles of y (the fixture's
    target_rule), trees, LEAF-major leaf values, staged raw approximants and
    class probabilities."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    cfg = json.loads(_read(os.path.join(fx, "multiclass_softmax/config.json")))
    model = json.loads(_read(os.path.join(fx, "multiclass_softmax/model.json")))
    X = np.load(os.path.join(fx, "inputs/numeric_tiny/X.npy"))
    y = np.load(os.path.join(fx, "inputs/numeric_tiny/y.npy"))
    cls = np.digitize(y, np.quantile(y, [1 / 3, 2 / 3])).astype(np.int32)
    K = int(cfg["approx_dimension"])
    trees = model["oblivious_trees"]
    depth = max(len(t["splits"]) for t in trees)
    sf = np.array([[s["float_feature_index"] for s in t["splits"]] for t in trees], dtype=np.int32)
    sv = np.array([[s["border"] for s in t["splits"]] for t in trees], dtype=np.float64)
    lv = np.array([t["leaf_values"] for t in trees], dtype=np.float64).reshape(len(trees), 1 << depth, K)
    n = X.shape[0]
    p = cfg["params"]
    params = {"loss": "MultiClass", "n_classes": K, "depth": int(p["depth"]), "iterations": int(p["iterations"]),
              "learning_rate": float(p["learning_rate"]), "l2_leaf_reg": float(p["l2_leaf_reg"]),
              "score_function": p["score_function"], "bootstrap_type": p["bootstrap_type"],
              "random_seed": int(p["random_seed"]), "border_count": 254, "border_type": "GreedyLogSum"}
    np.savez_compressed(os.path.join(OUT, "multiclass_softmax.npz"), X=X.astype(np.float32), target_class=cls,
                        split_feature=sf, split_border=sv, leaf_values=lv,
                        staged=np.load(os.path.join(fx, "multiclass_softmax/staged.npy")).reshape(len(trees), n, K),
                        probabilities=np.load(os.path.join(fx, "multiclass_softmax/predictions.npy")).reshape(n, K),
                        params=np.array(json.dumps(params)))
    return "multiclass_softmax"


def multi_output_fixtures(ref):
    """Upstream MultiClassOneVsAll, MultiLogloss, MultiCrossEntropy and
    RMSEWithUncertainty fixtures on numeric_tiny (Newton leaves).  Labels are stored
    as the dim-major [K, n] matrix each fit consumes: OneVsAll's one-hot of the
    digitized classes (the multiclass_softmax rule); for the two label losses
    the nested thresholds y > quantile(y, [.25, .5, .75]) that the reference's
    multilabel_oracle_test.rs:67-85 derives (the configs' target_rule text
    names another rule, which does not reproduce upstream's staged values)."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    X = np.load(os.path.join(fx, "inputs/numeric_tiny/X.npy"))
    y = np.load(os.path.join(fx, "inputs/numeric_tiny/y.npy"))
    n = X.shape[0]
    out = {"X": X.astype(np.float32)}
    for sc in ("multiclass_onevsall", "multilogloss", "multicrossentropy", "rmse_uncertainty"):
        cfg = json.loads(_read(os.path.join(fx, sc, "config.json")))
        model = json.loads(_read(os.path.join(fx, sc, "model.json")))
        K = int(cfg["approx_dimension"])
        if sc == "multiclass_onevsall":
            cls = np.digitize(y, np.quantile(y, [1 / 3, 2 / 3]))
            labels = (np.arange(K)[:, None] == cls[None, :]).astype(np.float64)
        elif sc == "rmse_uncertainty":  # the raw target; K = 2 is [mean, log-scale]
            labels = y[None, :].astype(np.float64)
        else:
            labels = np.vstack([y > np.quantile(y, q) for q in (0.25, 0.5, 0.75)]).astype(np.float64)
        trees = model["oblivious_trees"]
        depth = max(len(t["splits"]) for t in trees)
        p = cfg["params"]
        params = {"loss": cfg["loss_function"], "approx_dimension": K, "depth": int(p["depth"]),
                  "iterations": int(p["iterations"]), "learning_rate": float(p["learning_rate"]),
                  "l2_leaf_reg": float(p["l2_leaf_reg"]), "score_function": p["score_function"],
                  "leaf_estimation_method": p["leaf_estimation_method"], "border_count": 254,
                  "border_type": "GreedyLogSum"}
        out[f"{sc}__labels"] = labels
        out[f"{sc}__split_feature"] = np.array([[s["float_feature_index"] for s in t["splits"]] for t in trees],
                                               dtype=np.int32)
        out[f"{sc}__split_border"] = np.array([[s["border"] for s in t["splits"]] for t in trees], dtype=np.float64)
        out[f"{sc}__leaf_values"] = np.array([t["leaf_values"] for t in trees],
                                             dtype=np.float64).reshape(len(trees), 1 << depth, K)
        out[f"{sc}__staged"] = np.load(os.path.join(fx, sc, "staged.npy")).reshape(len(trees), n, K)
        out[f"{sc}__probabilities"] = np.load(os.path.join(fx, sc, "predictions.npy")).reshape(n, K)
        out[f"{sc}__params"] = np.array(json.dumps(params))
    np.savez_compressed(os.path.join(OUT, "multi_output.npz"), **out)
    return "multi_output"


def ranking_fixtures(ref):
    """Upstream QueryRMSE / PairLogit / PairLogitPairwise / QuerySoftMax / LambdaMart fixtures on the reference's frozen ranking
    corpus (12 objects, 5 contiguous groups, 7 explicit pairs): inputs, group
    offsets, pairs, and per loss the trees, leaf values and staged approximants."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures/ranking_corpus")
    gid = np.load(os.path.join(fx, "inputs/group_id.npy"))
    offsets = np.concatenate([[0], np.flatnonzero(np.diff(gid)) + 1, [gid.size]]).astype(np.int64)
    arrays = dict(X=np.load(os.path.join(fx, "inputs/X.npy")).astype(np.float32),
                  y=np.load(os.path.join(fx, "inputs/y.npy")).astype(np.float64), group_offsets=offsets,
                  pairs=np.load(os.path.join(fx, "inputs/pairs.npy")).astype(np.int64))
    losses = []
    for loss in ("QueryRMSE", "PairLogit", "PairLogitPairwise", "QuerySoftMax", "LambdaMart", "YetiRank",
                 "StochasticRank", "YetiRankPairwise"):
        d = {"YetiRank": "yetirank", "StochasticRank": "stochasticrank",
             "YetiRankPairwise": "yetirank_pairwise"}.get(loss, loss)
        cfg = json.loads(_read(os.path.join(fx, d, "config.json")))
        model = json.loads(_read(os.path.join(fx, d, "model.json")))
        mparams = model["model_info"].get("params")
        mparams = json.loads(mparams) if isinstance(mparams, str) else (mparams or {})
        tlo = mparams.get("tree_learner_options", {})
        l2 = float(tlo.get("l2_leaf_reg", 3.0))
        lf = mparams.get("loss_function", {}).get("params", {})
        trees = model["oblivious_trees"]
        arrays[f"{loss}__split_feature"] = np.array([[s["float_feature_index"] for s in t["splits"]] for t in trees],
                                                    dtype=np.int32)
        arrays[f"{loss}__split_border"] = np.array([[s["border"] for s in t["splits"]] for t in trees])
        arrays[f"{loss}__leaf_values"] = np.array([t["leaf_values"] for t in trees], dtype=np.float64)
        arrays[f"{loss}__staged"] = np.load(os.path.join(fx, d, "staged.npy")).reshape(len(trees), -1)
        arrays[f"{loss}__params"] = np.array(json.dumps({
            "depth": int(cfg["depth"]), "iterations": int(cfg["iterations"]),
            "learning_rate": float(cfg["learning_rate"]), "l2_leaf_reg": l2,
            "random_seed": int(cfg["random_seed"]), "leaf_estimation_method": tlo.get("leaf_estimation_method"),
            "softmax_lambda": float(lf.get("lambda", 0.01)), "softmax_beta": float(lf.get("beta", 1.0)),
            "lambdamart_sigma": float(lf.get("sigma", 1.0)), "lambdamart_top": int(lf.get("top", -1)),
            "lambdamart_norm": str(lf.get("norm", "true")).lower() == "true",
            "lambdamart_metric": str(lf.get("metric", "NDCG")),
            "yeti_permutations": int(lf.get("permutations", 10)), "yeti_decay": float(lf.get("decay", 0.85)),
            "srank_metric": str(lf.get("metric", "NDCG")), "srank_sigma": float(lf.get("sigma", 1.0)),
            "srank_mu": float(lf.get("mu", 0.0)), "srank_num_estimations": int(lf.get("num_estimations", 1))}))
        losses.append(loss)
    # YetiRank's instrumented sampler log: one 3-document group (raw approx
    # [0.5, -0.3, 0.1], relevances [2, 0, 1], 10 permutations, decay 0.85,
    # random_seed 0, the reference's yetirank_oracle_test.rs:213-260), and the
    # trainer's per-tree recalc seeds (update_pairs events: deriv, learning
    # fold, leaf values per tree)
    ev = [json.loads(l) for l in _read(os.path.join(fx, "yetirank/yetirank_rng_groundtruth.jsonl")).splitlines()
          if l.strip()]
    arrays["yeti_gt_query_seed"] = np.array([e["seed"] for e in ev if e["event"] == "query_seed"], dtype=np.uint64)
    arrays["yeti_gt_competitors"] = np.array([[e["winner"], e["loser"], e["weight"]] for e in ev
                                              if e["event"] == "competitor"], dtype=np.float64)
    arrays["yeti_gt_sorted_orders"] = np.array([e["order"] for e in ev if e["event"] == "sorted_order"],
                                               dtype=np.int64)
    tr = [json.loads(l) for l in _read(os.path.join(
        fx, "yetirank_pairwise/yetirank_pairwise_tree_rng_groundtruth.jsonl")).splitlines() if l.strip()]
    arrays["yeti_gt_recalc_seeds"] = np.array([e["random_seed"] for e in tr if e["event"] == "update_pairs"],
                                              dtype=np.uint64).reshape(-1, 3)
    # StochasticRank's trainer noise log: per tree and phase each group's
    # std_normal stream seeded with the recalc base + the group index
    sn = [json.loads(l) for l in _read(os.path.join(
        fx, "stochasticrank/stochasticrank_pertree_noise_groundtruth.jsonl")).splitlines() if l.strip()]
    arrays["srank_gt_noise_seed"] = np.array([e["seed"] for e in sn], dtype=np.uint64)
    arrays["srank_gt_noise"] = np.array([[e["sample"], e["doc"], e["count"], e["noise"]] for e in sn])
    np.savez_compressed(os.path.join(OUT, "ranking_corpus.npz"), **arrays)
    return ["ranking_corpus/" + l for l in losses]


def one_hot_fixtures(ref):
    """Upstream one-hot categorical fixtures: the reference's CityHash vectors
    (crates/cb-oracle/fixtures/cat_hash: CalcCatFeatureHash and its 64-bit
    precursor per string, per-object hashes and first-seen perfect-hash bins)
    and the two one_hot_train Logloss fits (float columns, categorical labels,
    the model's float borders, per-tree splits -- one-hot splits by hash --,
    leaf values and predictions)."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    ch = json.loads(_read(os.path.join(fx, "cat_hash/config.json")))
    keys = sorted(ch["string_to_ui32"])
    arrays = {"hash_strings": np.array(keys),
              "hash_ui32": np.array([ch["string_to_ui32"][k] for k in keys], dtype=np.uint64),
              "hash_ui64": np.array([int(ch["string_to_ui64_precursor"][k]) for k in keys], dtype=np.uint64),
              "hash_c0_order": np.array(ch["c0_first_seen_order"]),
              "hash_c1_order": np.array(ch["c1_first_seen_order"]),
              "hash_per_object": np.load(os.path.join(fx, "cat_hash/cat_hashes.npy")).astype(np.uint64),
              "hash_bins": np.load(os.path.join(fx, "cat_hash/perfect_hash_bins.npy")).astype(np.int64)}
    names = []
    for sc in ("default_binary", "multi"):
        d = os.path.join(fx, "one_hot_train", sc)
        cfg = json.loads(_read(os.path.join(d, "config.json")))
        model = json.loads(_read(os.path.join(d, "model.json")))
        cc = json.loads(_read(os.path.join(d, "cat_cols.json")))
        p = cfg["params"]
        arrays[f"{sc}__X"] = np.load(os.path.join(d, "X_float.npy")).astype(np.float32)
        arrays[f"{sc}__y"] = np.load(os.path.join(d, "y.npy")).astype(np.float64)
        arrays[f"{sc}__cat"] = np.array(cc["columns"])
        arrays[f"{sc}__predictions"] = np.load(os.path.join(d, "predictions.npy")).astype(np.float64)
        ff = model["features_info"]["float_features"]
        for f in ff:
            arrays[f"{sc}__borders{f['feature_index']}"] = np.array(f.get("borders") or [], dtype=np.float64)
        trees = model["oblivious_trees"]
        kind, feat, val = [], [], []
        for t in trees:
            kind.append([0 if s["split_type"] == "FloatFeature" else 1 for s in t["splits"]])
            feat.append([s.get("float_feature_index", s.get("cat_feature_index")) for s in t["splits"]])
            val.append([s["border"] if s["split_type"] == "FloatFeature" else float(s["value"] & 0xffffffff)
                        for s in t["splits"]])
        arrays[f"{sc}__split_kind"] = np.array(kind, dtype=np.int32)
        arrays[f"{sc}__split_feature"] = np.array(feat, dtype=np.int32)
        arrays[f"{sc}__split_value"] = np.array(val, dtype=np.float64)
        arrays[f"{sc}__leaf_values"] = np.array([t["leaf_values"] for t in trees], dtype=np.float64)
        arrays[f"{sc}__params"] = np.array(json.dumps({
            "depth": int(p["depth"]), "iterations": int(p["iterations"]), "learning_rate": float(p["learning_rate"]),
            "l2_leaf_reg": float(p["l2_leaf_reg"]), "loss": p["loss_function"], "score_function": p["score_function"],
            "leaf_estimation_method": p["leaf_estimation_method"], "one_hot_max_size": int(p["one_hot_max_size"]),
            "n_float": len(ff)}))
        names.append("one_hot_train/" + sc)
    np.savez_compressed(os.path.join(OUT, "one_hot.npz"), **arrays)
    return names


def model_json_fixtures(ref):
    """Upstream model.json documents (the reference's JSON model format,
    crates/cb-model/src/json.rs) of five fixtures, as text: the regression and
    binary skeletons, both NaN modes, and the 3-class softmax model."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    docs = {"regression_skeleton": "regression_skeleton/model.json", "binclf_skeleton": "binclf_skeleton/model.json",
            "nan_mode_Max": "nan_mode/model_Max.json", "nan_mode_Min": "nan_mode/model_Min.json",
            "multiclass_softmax": "multiclass_softmax/model.json"}
    arrays = {k: np.array(json.dumps(json.loads(_read(os.path.join(fx, v))))) for k, v in docs.items()}
    np.savez_compressed(os.path.join(OUT, "model_json.npz"), **arrays)
    return ["model_json/" + k for k in docs]


def cbm_fixtures(ref):
    """Upstream .cbm model files (the reference's binary model format,
    crates/cb-model/src/cbm.rs) as raw bytes, with what pins them: the same
    model's model.json where upstream wrote one, and upstream's predictions
    on the fixture rows (model_sum).  The one-hot fits' rows, categories and
    predictions are in one_hot.npz."""
    fx = os.path.join(ref, "crates/cb-oracle/fixtures")
    files = {"model_sum_m0": ("model_sum/m0.cbm", None), "model_sum_m1": ("model_sum/m1.cbm", None),
             "mae": ("fstr_loss_change/mae_model.cbm", "fstr_loss_change/mae_model.json"),
             "partial_dependence": ("partial_dependence/model.cbm", "partial_dependence/model.json"),
             "staged_predict": ("staged_predict/model.cbm", None),
             "one_hot_default_binary": ("one_hot_train/default_binary/model.cbm",
                                        "one_hot_train/default_binary/model.json"),
             "one_hot_multi": ("one_hot_train/multi/model.cbm", "one_hot_train/multi/model.json")}
    arrays = {}
    for name, (cbm, js) in files.items():
        with open(os.path.join(fx, cbm), "rb") as f:
            arrays[name + "__cbm"] = np.frombuffer(f.read(), dtype=np.uint8)
        if js:
            arrays[name + "__json"] = np.array(json.dumps(json.loads(_read(os.path.join(fx, js)))))
    arrays["model_sum__X"] = np.load(os.path.join(fx, "model_sum/X.npy")).astype(np.float32)
    for m in ("m0", "m1"):
        arrays[f"model_sum__expected_{m}"] = np.load(os.path.join(fx, f"model_sum/expected_{m}.npy")).astype(np.float64)
    np.savez_compressed(os.path.join(OUT, "model_cbm.npz"), **arrays)
    return ["model_cbm/" + k for k in files]


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CB_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        sys.exit("usage: make_golden.py <reference checkout>")
    with open(os.path.join(OUT, "scalar_vectors.json"), "w") as f:
        json.dump(scalar_vectors(ref), f, indent=1)
    border_cells = border_fixtures(ref)
    written = e2e_fixtures(ref)
    written.append(multiclass_fixture(ref))
    written.append(multi_output_fixtures(ref))
    written += ranking_fixtures(ref)
    written += one_hot_fixtures(ref)
    written += model_json_fixtures(ref)
    written += cbm_fixtures(ref)
    with open(os.path.join(OUT, "MANIFEST.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "origin": "upstream CatBoost 1.2.10 fixtures committed under the reference's "
                             "crates/cb-oracle/fixtures (thread_count=1, random_strength per scenario)",
                   "scenarios": written, "border_cells": border_cells}, f, indent=1)
    print("wrote", len(written), "scenarios")


if __name__ == "__main__":
    main()
