"""Throughput of the multi-output, ranking and scale workloads (BASELINE
configs 3, 4 and 5), run by `bench.py --config N`.

Each prints one JSON line with the config-2 bench's keys where they apply:
trees/s over K timed trees after W warm-up trees, by the host clock around
synchronous grow calls (each call returns the grown tree to the host, so the
clock spans the device work and the result copy), on seeded synthetic data of
the config's shapes and distributions (no public dataset is named).

- config 3: MultiClass, 10 classes, 2M rows x 100 N(0,1) float features plus
  20 categorical int features (Zipf s = 1.2, cardinality 5-200) as one-hot
  features, class = argmax of 10 random linear scores + Gumbel noise, depth 6.
  The reference rejects one-hot features with a bootstrap, so the one-hot
  variant runs with bootstrap No and the Bernoulli (subsample 0.66) variant
  on the float features only (`--variant onehot|bernoulli`).
- config 4: grouped ranking, 1M documents in query groups of uniform size
  20-120, 136 features (half log-normal counts, half U(0,1) ratios),
  border_count 128, relevance 0-4 from a noisy linear score per query,
  depth 6; YetiRank (pairs sampled on the device) or PairLogit (pairs of
  differently relevant documents, at most 200 per query), each also with
  the pairwise scorer and Cholesky pairwise leaves
  (`--variant yetirank|pairlogit|yetirankpairwise|pairlogitpairwise`).
- config 5: RMSE, 50M rows x 500 N(0,1) features, border_count 128, sparse
  linear target + noise, depth 10, MVS subsample 0.8, on the scalar session
  (the same path as config 2); document-sharded under torchrun.
"""
from __future__ import annotations

import json
import os
import time

import numpy as np

import catboost_rs_b200 as cb

FMIN = float(np.finfo(np.float32).min)


def _borders(X, border_count, seed, nan_sentinel=False):
    g = np.random.default_rng([seed, 7])
    n = X.shape[1]
    idx = g.choice(n, size=min(n, 200_000), replace=False)
    out = []
    for f in range(X.shape[0]):
        q = np.quantile(X[f, idx].astype(np.float64), np.linspace(0, 1, border_count + 1)[1:-1])
        b = np.unique(q.astype(np.float32).astype(np.float64))
        out.append(np.concatenate([[FMIN], b]) if nan_sentinel else b)
    return out


def config3_data(seed=0, n=2_000_000, F=100, n_cat=20, K=10):
    g = np.random.default_rng([seed, 3])
    X = g.standard_normal((F, n), dtype=np.float32)
    cats = []
    card = g.integers(5, 201, size=n_cat)
    for c in range(n_cat):
        k = np.arange(1, card[c] + 1, dtype=np.float64)
        p = k ** -1.2
        cats.append(g.choice(card[c], size=n, p=p / p.sum()).astype(np.int64))
    W = g.standard_normal((F, K)) * (g.random((F, 1)) < 0.3)
    score = X.T.astype(np.float64) @ W
    for c in range(4):  # a few categorical effects
        eff = g.standard_normal((card[c], K)) * 0.5
        score += eff[cats[c]]
    score += g.gumbel(size=score.shape)
    y = np.argmax(score, axis=1).astype(np.float64)
    return X, cats, y


def config4_data(seed=0, n=1_000_000, F=136):
    g = np.random.default_rng([seed, 4])
    sizes = []
    tot = 0
    while tot < n:
        s = int(g.integers(20, 121))
        s = min(s, n - tot)
        sizes.append(s)
        tot += s
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    h = F // 2
    X = np.empty((F, n), dtype=np.float32)
    X[:h] = np.floor(g.lognormal(1.0, 1.2, size=(h, n))).astype(np.float32)
    X[h:] = g.random((F - h, n), dtype=np.float32)
    w = g.standard_normal(F) * (g.random(F) < 0.2)
    z = w @ np.log1p(np.abs(X.astype(np.float64)))
    rel = np.empty(n)
    for q in range(len(sizes)):
        a, b = offsets[q], offsets[q + 1]
        s = z[a:b] + g.standard_normal(b - a)
        edges = np.quantile(s, [0.4, 0.7, 0.88, 0.97])
        rel[a:b] = np.searchsorted(edges, s)
    return X, rel, offsets


def config4_pairs(rel, offsets, seed=0, cap=200):
    g = np.random.default_rng([seed, 41])
    out = []
    for q in range(len(offsets) - 1):
        a, b = int(offsets[q]), int(offsets[q + 1])
        r = rel[a:b]
        i, j = np.nonzero(r[:, None] > r[None, :])
        if i.size > cap:
            keep = g.choice(i.size, size=cap, replace=False)
            i, j = i[keep], j[keep]
        out.append(np.stack([i + a, j + a], axis=1))
    return np.concatenate(out).astype(np.int64)


def _line(metric, value, steps, warmup, sec, workload, extra):
    d = {"metric": metric, "value": value, "unit": "trees/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
         "ms_per_step": 1e3 * sec / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
         "dtype": "int64", "data": "synthetic (seeded, the config's shapes and distributions)",
         "config": dict(workload=workload, **extra), "roofline": None, "cpu_baseline": None, "e2e": None}
    print(json.dumps(d), flush=True)


def run_config3(args):
    variant = args.variant or "onehot"
    X, cats, y = config3_data(args.seed)
    F, n = X.shape
    K = 10
    borders = _borders(X, 128, args.seed)
    cols = [np.ascontiguousarray(X[f]) for f in range(F)]
    rt = cb.B200MultiRuntime()
    boot = "No" if variant == "onehot" else "Bernoulli"
    cfg = cb.DeviceTrainConfig(bootstrap_type=boot, sample_rate=0.66, rng_seed=0, bias=0.0, sample_from_host=False)
    cat_bins = []
    if variant == "onehot":
        for c in cats:
            b, _ = cb.boosting.perfect_hash_bins(c.tolist())
            cat_bins.append(b)
    nb = max(len(b) for b in borders) + 1
    lr = float(np.float32(0.1))
    assert rt.begin_device_training_raw("MultiClass", 6, True, 1, "Cosine", cols, borders, None, n, F, nb, lr, 3.0,
                                        cfg, approx_dim=K, cat_columns=cat_bins), rt.decline_reason
    fam = ("MultiOutput", None, K)
    try:
        for _ in range(args.warmup):
            rt.grow_tree_on_device(None, y, [], family=fam, leaf_of_bytes=0, resident_approx=True)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            rt.grow_tree_on_device(None, y, [], family=fam, leaf_of_bytes=0, resident_approx=True)
        sec = time.perf_counter() - t0
    finally:
        rt.end_device_training()
    _line("trees/sec at 2M x 100 (+20 one-hot) MultiClass-10 depth 6", args.steps / sec, args.steps, args.warmup,
          sec, f"config3 ({variant}): MultiClass K=10, 2M rows x 100 N(0,1) f32"
          + (" + 20 one-hot categorical (Zipf 1.2, cardinality 5-200), bootstrap No" if variant == "onehot"
             else ", Bernoulli subsample 0.66 (no categorical: the reference rejects one-hot with a bootstrap)")
          + ", border_count 128, depth 6, lr 0.1, l2 3, Cosine",
          {"rows": n, "features": F + (len(cats) if variant == "onehot" else 0), "depth": 6, "classes": K,
           "timing": "host clock around synchronous grow calls"})


def run_config4(args):
    variant = args.variant or "yetirank"
    X, rel, offsets = config4_data(args.seed)
    F, n = X.shape
    borders = _borders(X, 128, args.seed)
    cols = [np.ascontiguousarray(X[f]) for f in range(F)]
    loss = {"yetirank": "YetiRank", "pairlogit": "PairLogit", "pairlogitpairwise": "PairLogitPairwise",
            "yetirankpairwise": "YetiRankPairwise"}[variant]
    pairs = config4_pairs(rel, offsets, args.seed) if variant.startswith("pairlogit") else None
    rt = cb.B200MultiRuntime()
    cfg = cb.DeviceTrainConfig(bootstrap_type="No", rng_seed=0, bias=0.0)
    nb = max(len(b) for b in borders) + 1
    lr = float(np.float32(0.1))
    assert rt.begin_ranking_raw(loss, 6, True, 1, "Cosine", cols, borders, None, n, F, nb, lr, 3.0, cfg,
                                offsets, pairs=pairs, l2_leaf_reg=3.0 if loss.endswith("Pairwise") else None), \
        rt.decline_reason
    try:
        for _ in range(args.warmup):
            rt.grow_tree_on_device(None, rel, [], leaf_of_bytes=0, resident_approx=True)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            rt.grow_tree_on_device(None, rel, [], leaf_of_bytes=0, resident_approx=True)
        sec = time.perf_counter() - t0
    finally:
        rt.end_device_training()
    _line(f"trees/sec at 1M docs x 136 {loss} depth 6", args.steps / sec, args.steps, args.warmup, sec,
          f"config4 ({variant}): {loss}, 1M documents in {len(offsets) - 1} query groups of 20-120, 136 features "
          "(log-normal counts + U(0,1)), relevance 0-4, border_count 128, depth 6, lr 0.1, l2 3"
          + (f", {len(pairs)} pairs (<= 200 per query)" if pairs is not None else ", pairs sampled on the device"),
          {"rows": n, "features": F, "depth": 6, "groups": len(offsets) - 1,
           "timing": "host clock around synchronous grow calls"})
