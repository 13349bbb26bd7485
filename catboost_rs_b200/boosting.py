"""The boosting loop on top of the B200 runtime, mirroring cb-train's device
branch (crates/cb-train/src/boosting.rs:6532-7300) for the covered regime:
SymmetricTree, RMSE / Logloss / CrossEntropy, Plain, Cosine / L2, Gradient
leaves, bootstrap No / Bayesian / Bernoulli / MVS.

The session keeps the approximant and the bootstrap resident on the device and
replays the main RNG stream's draw accounting itself (PRE draws, bootstrap,
per-level replay, POST draws), so trees match the CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from .runtime import B200MultiRuntime, B200Runtime, DeviceTrainConfig, apply_oblivious, flatten_oblivious


@dataclass
class FitParams:
    loss: str = "RMSE"
    depth: int = 6
    iterations: int = 100
    learning_rate: float = 0.1
    l2_leaf_reg: float = 3.0
    score_function: str = "Cosine"
    bootstrap_type: str = "No"
    subsample: float = 0.8
    bagging_temperature: float = 1.0
    random_seed: int = 0
    boost_from_average: bool = True
    softmax_lambda: float = 0.01  # QuerySoftMax:lambda
    softmax_beta: float = 1.0     # QuerySoftMax:beta
    lambdamart_sigma: float = 1.0  # LambdaMart:sigma
    lambdamart_top: int = -1       # LambdaMart:top (-1: the whole group)
    lambdamart_norm: bool = True   # LambdaMart:norm
    lambdamart_metric: str = "NDCG"
    yeti_permutations: int = 10    # YetiRank:permutations
    yeti_decay: float = 0.85       # YetiRank:decay
    srank_metric: str = "DCG"      # StochasticRank:metric (DCG / NDCG)
    srank_sigma: float = 1.0
    srank_mu: float = 0.0
    srank_num_estimations: int = 1
    leaf_estimation_method: str = "Gradient"  # "Exact" for MAE / Quantile
    quantile_alpha: float = 0.5    # Quantile:alpha
    quantile_delta: float = 1e-6   # Quantile:delta


@dataclass
class ObliviousModel:
    """Per-tree splits (feature, border index; level l is leaf bit l), the
    learning-rate scaled leaf values, the borders and the bias."""
    borders: list
    split_feature: np.ndarray
    split_bin: np.ndarray
    leaf_values: np.ndarray
    bias: float
    staged: Optional[np.ndarray] = None
    stage_timing: list = field(default_factory=list)
    leaf_weights: Optional[np.ndarray] = None  # [T, 2^depth] when known (model.json)

    def split_borders(self) -> np.ndarray:
        return np.array([[self.borders[f][b] for f, b in zip(rf, rb)]
                         for rf, rb in zip(self.split_feature, self.split_bin)])

    def predict(self, X, device: int = 0) -> np.ndarray:
        """Raw approximant for rows of X (f32 [n, F]) through the device apply
        (Model::predict_raw_on_device): float value > border passes, NaN passes
        only on nan_mode=Max features (border list ends with f32::MAX)."""
        X = np.asarray(X, dtype=np.float32)
        fmax = np.float64(np.finfo(np.float32).max)
        nan_above = np.array([len(b) > 0 and b[-1] == fmax for b in self.borders], dtype=np.uint8)
        flat = flatten_oblivious(self.split_feature, self.split_borders(), self.leaf_values)
        return apply_oblivious(np.ascontiguousarray(X.T), flat, self.bias, nan_above, device)


def seq_sum(v) -> float:
    """Strict left-to-right f64 sum (cb_core::sum_f64): numpy's cumsum is sequential."""
    v = np.asarray(v, dtype=np.float64)
    return float(np.cumsum(v)[-1]) if v.size else 0.0


def starting_approx(p: FitParams, target) -> float:
    """boosting.rs:1871: mean target for RMSE with boost_from_average, else 0."""
    if p.boost_from_average and p.loss == "RMSE" and len(target):
        return seq_sum(target) / len(target)
    return 0.0


def fit(float_columns: Sequence[np.ndarray], borders: Sequence[Sequence[float]], target,
        params: FitParams, weights=None, *, staged: bool = False, device: int = 0,
        placement: Optional[dict] = None, profile: bool = False,
        bias: Optional[float] = None, sum_weights: Optional[float] = None) -> ObliviousModel:
    """Fit on raw f32 columns with fixed borders (device quantization).

    `placement` = {rank, world_size, row_offset, n_total, nccl_unique_id} for a
    document-sharded fit (one process per GPU); `bias` / `sum_weights` are then
    the GLOBAL starting approximant and weight total.
    """
    p = params
    cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
    F = len(cols)
    n = cols[0].size if F else 0
    t = np.ascontiguousarray(target, dtype=np.float64)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    pl = placement or {}
    n_total = pl.get("n_total", n)
    # scale_l2_reg (leaf.rs:177) uses the GLOBAL weight sum and row count
    if sum_weights is not None:
        sw = sum_weights
    elif w is not None:
        if n != n_total:
            raise ValueError("a sharded weighted fit needs sum_weights (the global weight sum)")
        sw = seq_sum(w)
    else:
        sw = float(n_total)
    scaled_l2 = p.l2_leaf_reg * (sw / n_total) if n_total else p.l2_leaf_reg
    b0 = bias if bias is not None else starting_approx(p, t)
    # upstream stores the learning rate as f32, and cb-train hands the narrowed
    # value to the seam and to normalize_leaf_values (boosting.rs:4958)
    lr = float(np.float32(p.learning_rate))
    n_bins = max(len(b) for b in borders) + 1
    cfg = DeviceTrainConfig(bootstrap_type=p.bootstrap_type, sample_rate=p.subsample,
                            rng_seed=p.random_seed, bias=b0, sample_from_host=False,
                            bagging_temperature=p.bagging_temperature, device=device,
                            rank=pl.get("rank", 0), world_size=pl.get("world_size", 1),
                            row_offset=pl.get("row_offset", 0), n_total=n_total,
                            nccl_unique_id=pl.get("nccl_unique_id"),
                            exact_leaf=p.leaf_estimation_method == "Exact", quantile_alpha=p.quantile_alpha,
                            quantile_delta=p.quantile_delta)
    rt = B200Runtime()
    ok = rt.begin_device_training_raw(p.loss, p.depth, True, 1, p.score_function, cols, borders, w,
                                      n, F, n_bins, lr, scaled_l2, cfg)
    if not ok:
        raise RuntimeError(f"device declined: {rt.decline_reason}")
    if profile:
        rt.set_profiling(True)
    T, D = p.iterations, p.depth
    sf = np.zeros((T, D), dtype=np.int32)
    sb = np.zeros((T, D), dtype=np.int32)
    lv = np.zeros((T, 1 << D), dtype=np.float64)
    st = np.zeros((T, n), dtype=np.float64) if staged else None
    timings = []
    try:
        for it in range(T):
            tree = rt.grow_tree_on_device(None, t, [], leaf_of_bytes=0, resident_approx=True)
            for l, (f, b, _) in enumerate(tree.splits):
                sf[it, l], sb[it, l] = f, b
            lv[it] = tree.leaf_values * lr  # normalize_leaf_values
            if staged:
                st[it] = rt.resident_approx()
            if profile:
                timings.append(rt.timing().copy())
    finally:
        rt.end_device_training()
    return ObliviousModel([np.asarray(b, dtype=np.float64) for b in borders], sf, sb, lv, b0, st, timings)


@dataclass
class MultiClassModel:
    """Per-tree splits, the learning-rate scaled LEAF-major leaf blocks
    [T, 2^depth, K], the borders, and optionally the staged raw approximants
    [T, n, K] (object-major, upstream's staged_predict layout)."""
    borders: list
    split_feature: np.ndarray
    split_bin: np.ndarray
    leaf_values: np.ndarray
    staged: Optional[np.ndarray] = None
    cat_values: Optional[list] = None  # per one-hot feature, its categories in bin order
    leaf_weights: Optional[np.ndarray] = None  # [T, 2^depth] when known (model.json)

    def split_borders(self) -> np.ndarray:
        """Float splits' borders; NaN for one-hot splits (split_feature >= the float count)."""
        F = len(self.borders)
        return np.array([[self.borders[f][b] if f < F else np.nan for f, b in zip(rf, rb)]
                         for rf, rb in zip(self.split_feature, self.split_bin)])


def perfect_hash_bins(column):
    """The perfect-hash bins of one categorical column as the reference's quantizer assigns
    them: bin = the category's first-seen order.  Returns (uint32 bins [n], categories in bin
    order)."""
    index = {}
    out = np.empty(len(column), dtype=np.uint32)
    for i, v in enumerate(column):
        out[i] = index.setdefault(v, len(index))
    return out, list(index)


def fit_multiclass(float_columns: Sequence[np.ndarray], borders: Sequence[Sequence[float]], target_class,
                   n_classes: int, params: FitParams, weights=None, *, staged: bool = False,
                   device: int = 0, cat_columns=None, loss: str = "MultiClass") -> MultiClassModel:
    """Multi-output fit (Newton leaves) on raw f32 columns with fixed borders:
    cb-train's multi-output loop (boosting.rs:7400-8930 at approx_dimension K)
    over the device's multi-output arm.

    loss "MultiClass" (softmax, coupled Hessian solve) and "MultiClassOneVsAll"
    (per-class sigmoid) take class indices in target_class; "MultiLogloss"
    ({0, 1}) and "MultiCrossEntropy" ([0, 1]) take the [K, n] label matrix
    (dim-major, the reference's multilabel layout) with n_classes = K labels.
    The three diagonal losses solve each dimension's leaf on its own
    (boosting.rs:8323-8420).  cat_columns are one-hot categorical features
    (any hashable values; bins in first-seen order); they need bootstrap No,
    as upstream."""
    p = params
    cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
    F = len(cols)
    n = cols[0].size if F else (len(cat_columns[0]) if cat_columns else 0)
    y = np.ascontiguousarray(target_class, dtype=np.float64)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    sw = seq_sum(w) if w is not None else float(n)
    scaled_l2 = p.l2_leaf_reg * (sw / n) if n else p.l2_leaf_reg
    lr = float(np.float32(p.learning_rate))  # boosting.rs:4958
    K = int(n_classes)
    cfg = DeviceTrainConfig(bootstrap_type=p.bootstrap_type, sample_rate=p.subsample, rng_seed=p.random_seed,
                            bias=0.0, sample_from_host=False, bagging_temperature=p.bagging_temperature,
                            device=device)
    rt = B200MultiRuntime()
    n_bins = max([len(b) for b in borders] + [0]) + 1
    cat_bins, cat_values = [], []
    for col in (cat_columns or []):
        b, v = perfect_hash_bins(col)
        cat_bins.append(b)
        cat_values.append(v)
    ok = rt.begin_device_training_raw(loss, p.depth, True, 1, p.score_function, cols, borders, w, n, F,
                                      n_bins, lr, scaled_l2, cfg, approx_dim=K, cat_columns=cat_bins)
    if not ok:
        raise RuntimeError(f"device declined: {rt.decline_reason}")
    T, D = p.iterations, p.depth
    sf = np.zeros((T, D), dtype=np.int32)
    sb = np.zeros((T, D), dtype=np.int32)
    lv = np.zeros((T, 1 << D, K), dtype=np.float64)
    st = np.zeros((T, n, K), dtype=np.float64) if staged else None
    try:
        for it in range(T):
            tree = rt.grow_tree_on_device(None, y, [], family=("MultiOutput", None, K), leaf_of_bytes=0,
                                          resident_approx=True)
            for l, (f, b, _) in enumerate(tree.splits):
                sf[it, l], sb[it, l] = f, b
            lv[it] = tree.leaf_values.reshape(1 << D, K) * lr  # normalize_leaf_values
            if staged:
                st[it] = rt.resident_approx().T
    finally:
        rt.end_device_training()
    return MultiClassModel([np.asarray(b, dtype=np.float64) for b in borders], sf, sb, lv, st,
                           cat_values if cat_columns else None)


@dataclass
class RankingModel:
    """Per-tree splits and the normalised, learning-rate scaled leaf values
    [T, 2^depth] of a grouped-loss fit, plus the raw Newton deltas the seam
    returned and optionally the staged approximants [T, n]."""
    borders: list
    split_feature: np.ndarray
    split_bin: np.ndarray
    leaf_values: np.ndarray
    raw_leaf_values: np.ndarray
    staged: Optional[np.ndarray] = None

    def split_borders(self) -> np.ndarray:
        return np.array([[self.borders[f][b] for f, b in zip(rf, rb)]
                         for rf, rb in zip(self.split_feature, self.split_bin)])


def normalize_leaf_values(pairwise: bool, lr: float, leaf_weights, raw) -> np.ndarray:
    """cb-train's normalize_leaf_values (boosting.rs:2844-2880): pairwise losses
    subtract the document-weighted mean leaf value (empty leaves become 0),
    then every value is scaled by the learning rate."""
    v = np.array(raw, dtype=np.float64)
    if pairwise:
        total = seq_sum(leaf_weights)
        if abs(total) > 1e-9:
            avg = seq_sum(v * leaf_weights) / total
            v = np.where(np.abs(leaf_weights) > 1e-9, v - avg, 0.0)
    return v * lr


def fit_ranking(float_columns: Sequence[np.ndarray], borders: Sequence[Sequence[float]], target, group_offsets,
                params: FitParams, pairs=None, weights=None, *, staged: bool = False,
                device: int = 0, pair_weights=None) -> RankingModel:
    """QueryRMSE / QuerySoftMax / LambdaMart / YetiRank / StochasticRank /
    PairLogit / PairLogitPairwise fit (params.loss) on raw f32 columns with fixed borders:
    cb-train's grouped
    loop (pointwise histograms with Newton or, for QuerySoftMax, Gradient
    leaves; or pairwise scoring and Cholesky leaves) over the device's ranking
    arm; leaf normalisation on the host as cb-train does it.  pair_weights
    (one per pair, default 1) weight PairLogit's pairs."""
    p = params
    cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
    F = len(cols)
    n = cols[0].size if F else 0
    y = np.ascontiguousarray(target, dtype=np.float64)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    sw = seq_sum(w) if w is not None else float(n)
    scaled_l2 = p.l2_leaf_reg * (sw / n) if n else p.l2_leaf_reg
    lr = float(np.float32(p.learning_rate))  # boosting.rs:4958
    cfg = DeviceTrainConfig(bootstrap_type="No", rng_seed=p.random_seed, bias=0.0, device=device)
    rt = B200MultiRuntime()
    n_bins = max(len(b) for b in borders) + 1
    ok = rt.begin_ranking_raw(p.loss, p.depth, True, 1, p.score_function, cols, borders, w, n, F, n_bins, lr,
                              scaled_l2, cfg, group_offsets, pairs, l2_leaf_reg=p.l2_leaf_reg,
                              softmax_lambda=p.softmax_lambda, softmax_beta=p.softmax_beta,
                              lambdamart_sigma=p.lambdamart_sigma, lambdamart_top=p.lambdamart_top,
                              lambdamart_norm=p.lambdamart_norm, lambdamart_metric=p.lambdamart_metric,
                              yeti_permutations=p.yeti_permutations, yeti_decay=p.yeti_decay,
                              srank_metric=p.srank_metric, srank_sigma=p.srank_sigma, srank_mu=p.srank_mu,
                              srank_num_estimations=p.srank_num_estimations, pair_weights=pair_weights)
    if not ok:
        raise RuntimeError(f"device declined: {rt.decline_reason}")
    T, D = p.iterations, p.depth
    L = 1 << D
    sf = np.zeros((T, D), dtype=np.int32)
    sb = np.zeros((T, D), dtype=np.int32)
    lv = np.zeros((T, L), dtype=np.float64)
    raw = np.zeros((T, L), dtype=np.float64)
    st = np.zeros((T, n), dtype=np.float64) if staged else None
    doc_w = w if w is not None else np.ones(n)
    try:
        for it in range(T):
            tree = rt.grow_tree_on_device(None, y, [], leaf_of_bytes=2, resident_approx=True)
            for l, (f, b, _) in enumerate(tree.splits):
                sf[it, l], sb[it, l] = f, b
            raw[it] = tree.leaf_values
            leaf_w = np.bincount(tree.leaf_of.astype(np.int64), weights=doc_w, minlength=L)
            lv[it] = normalize_leaf_values(p.loss in ("PairLogit", "PairLogitPairwise", "YetiRank", "YetiRankPairwise"),
                                           lr, leaf_w,
                                           tree.leaf_values)
            if staged:
                st[it] = rt.resident_approx()[0]
    finally:
        rt.end_device_training()
    return RankingModel([np.asarray(b, dtype=np.float64) for b in borders], sf, sb, lv, raw, st)
