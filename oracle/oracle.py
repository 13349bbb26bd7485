"""ctypes bindings for liboracle.so, the C restatement of catboost_rs's CPU path.

TEST INFRASTRUCTURE ONLY -- the parity checker and the timed CPU baseline.
Every function mirrors one routine of the reference (file:line given in
cb_oracle.c); nothing here is used by the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

LOSS = {"RMSE": 0, "Logloss": 1, "CrossEntropy": 2, "MAE": 3, "Quantile": 4}
BOOT = {"No": 0, "Bayesian": 1, "Bernoulli": 2, "MVS": 3}
SCORE = {"Cosine": 0, "L2": 1, "SolarL2": 2, "LOOL2": 5, "SatL2": 6}
BORDER_TYPE = {"Median": 0, "GreedyLogSum": 1, "UniformAndQuantiles": 2, "MinEntropy": 3,
               "MaxLogSum": 4, "Uniform": 5, "GreedyMinEntropy": 6}
NAN_MODE = {"Min": 0, "Max": 1, "Forbidden": 2}


def build() -> str:
    """Compile liboracle.so from cb_oracle.c (make, system gcc)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Rng(C.Structure):
    _fields_ = [("x1", C.c_uint64), ("c1", C.c_uint64), ("x2", C.c_uint64),
                ("c2", C.c_uint64), ("calls", C.c_uint64)]


class _TrainArgs(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("n_features", C.c_int32),
        ("bins_fm", C.c_void_p), ("border_counts", C.c_void_p),
        ("target", C.c_void_p), ("weights", C.c_void_p),
        ("loss", C.c_int32), ("depth", C.c_int32), ("iterations", C.c_int32),
        ("learning_rate", C.c_double), ("l2_leaf_reg", C.c_double),
        ("score_function", C.c_int32), ("bootstrap_type", C.c_int32),
        ("subsample", C.c_double), ("bagging_temperature", C.c_float),
        ("random_strength", C.c_double), ("random_seed", C.c_uint64),
        ("boost_from_average", C.c_int32), ("n_threads", C.c_int32),
        ("n_cat", C.c_int32), ("cat_bins_fm", C.c_void_p),
        ("exact_leaf", C.c_int32), ("quantile_alpha", C.c_double), ("quantile_delta", C.c_double),
    ]


class _TrainOut(C.Structure):
    _fields_ = [("split_feature", C.c_void_p), ("split_bin", C.c_void_p),
                ("tree_depth", C.c_void_p), ("leaf_values", C.c_void_p),
                ("staged", C.c_void_p), ("final_approx", C.c_void_p),
                ("bias", C.c_void_p), ("rng_calls", C.c_void_p), ("level_top2", C.c_void_p)]


class _MultiArgs(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("n_features", C.c_int32), ("bins_fm", C.c_void_p),
        ("border_counts", C.c_void_p), ("target_class", C.c_void_p), ("weights", C.c_void_p),
        ("n_classes", C.c_int32), ("depth", C.c_int32), ("iterations", C.c_int32),
        ("learning_rate", C.c_double), ("l2_leaf_reg", C.c_double), ("score_function", C.c_int32),
        ("bootstrap_type", C.c_int32), ("subsample", C.c_double), ("bagging_temperature", C.c_float),
        ("random_seed", C.c_uint64), ("n_threads", C.c_int32), ("n_cat", C.c_int32), ("cat_bins_fm", C.c_void_p),
        ("loss_kind", C.c_int32), ("target_matrix", C.c_void_p),
    ]


class _MultiOut(C.Structure):
    _fields_ = [("split_feature", C.c_void_p), ("split_bin", C.c_void_p), ("tree_depth", C.c_void_p),
                ("leaf_values", C.c_void_p), ("staged", C.c_void_p), ("final_approx", C.c_void_p)]


class _RankArgs(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("n_features", C.c_int32), ("bins_fm", C.c_void_p), ("border_counts", C.c_void_p),
        ("target", C.c_void_p), ("weights", C.c_void_p), ("loss", C.c_int32), ("n_groups", C.c_int32),
        ("group_offsets", C.c_void_p), ("n_pairs", C.c_int64), ("pair_winner", C.c_void_p),
        ("pair_loser", C.c_void_p), ("depth", C.c_int32), ("iterations", C.c_int32),
        ("learning_rate", C.c_double), ("l2_leaf_reg", C.c_double), ("score_function", C.c_int32),
        ("random_seed", C.c_uint64), ("softmax_lambda", C.c_double), ("softmax_beta", C.c_double),
        ("lambdamart_sigma", C.c_double), ("lambdamart_top", C.c_int64), ("lambdamart_norm", C.c_int32),
        ("yeti_permutations", C.c_int32), ("yeti_decay", C.c_double), ("srank_ndcg", C.c_int32),
        ("srank_sigma", C.c_double), ("srank_mu", C.c_double), ("srank_num_estimations", C.c_int32),
        ("lambdamart_no_op", C.c_int32), ("pair_weight", C.c_void_p),
    ]


class _RankOut(C.Structure):
    _fields_ = [("split_feature", C.c_void_p), ("split_bin", C.c_void_p), ("leaf_values", C.c_void_p),
                ("raw_leaf_values", C.c_void_p), ("staged", C.c_void_p)]


RANK_LOSS = {"QueryRMSE": 0, "PairLogit": 1, "PairLogitPairwise": 2, "QuerySoftMax": 3, "LambdaMart": 4, "YetiRank": 5, "StochasticRank": 6,
             "YetiRankPairwise": 7}


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.POINTER
        L.orc_rng_new.argtypes = [P(Rng), C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32]
        L.orc_rng_from_seed.argtypes = [P(Rng), C.c_uint64]
        L.orc_rng_gen.argtypes = [P(Rng)]
        L.orc_rng_gen.restype = C.c_uint64
        L.orc_rng_real1.argtypes = [P(Rng)]
        L.orc_rng_real1.restype = C.c_double
        L.orc_rng_advance.argtypes = [P(Rng), C.c_uint64]
        L.orc_rng_uniform.argtypes = [P(Rng), C.c_uint64]
        L.orc_rng_uniform.restype = C.c_uint64
        L.orc_std_normal.argtypes = [P(Rng)]
        L.orc_std_normal.restype = C.c_double
        L.orc_fast_logf.argtypes = [C.c_float]
        L.orc_fast_logf.restype = C.c_float
        L.orc_sum_f64.argtypes = [C.c_void_p, C.c_int64]
        L.orc_sum_f64.restype = C.c_double
        L.orc_quantize.argtypes = [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_compute_gradients.argtypes = [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                            C.c_void_p, C.c_void_p]
        L.orc_bootstrap.argtypes = [C.c_int32, C.c_void_p, C.c_int64, C.c_double, C.c_float,
                                    C.c_int32, C.c_double, P(Rng), C.c_void_p, C.c_void_p]
        L.orc_bootstrap.restype = C.c_int
        L.orc_build_histogram.argtypes = [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]
        L.orc_select_borders.argtypes = [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                         C.c_void_p, C.c_int64]
        L.orc_select_borders.restype = C.c_int64
        L.orc_border_sample_indices.argtypes = [C.c_int64, C.c_int64, P(C.c_int64)]
        L.orc_border_sample_indices.restype = C.c_void_p
        L.orc_apply_oblivious.argtypes = [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_double,
                                          C.c_void_p, C.c_void_p]
        L.orc_train_multiclass.argtypes = [P(_MultiArgs), P(_MultiOut)]
        L.orc_train_multiclass.restype = C.c_int
        L.orc_solve_symmetric_newton.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_double, C.c_void_p]
        L.orc_score_term.argtypes = [C.c_int32, C.c_double, C.c_double]
        L.orc_score_term.restype = C.c_double
        L.orc_cat_hash.argtypes = [C.c_char_p, C.c_size_t]
        L.orc_cat_hash.restype = C.c_uint32
        L.orc_city_hash64.argtypes = [C.c_char_p, C.c_size_t]
        L.orc_city_hash64.restype = C.c_uint64
        L.orc_train_ranking.argtypes = [P(_RankArgs), P(_RankOut)]
        L.orc_train_ranking.restype = C.c_int
        L.orc_yeti_sample_pairs.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_double, C.c_int32, C.c_double,
                                            C.c_uint64, C.c_void_p]
        L.orc_yeti_sample_pairs.restype = None
        L.orc_yeti_query_seeds.argtypes = [C.c_uint64, C.c_int32, C.c_void_p]
        L.orc_yeti_query_seeds.restype = None
        L.orc_yeti_recalc_seeds.argtypes = [C.c_uint64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]
        L.orc_yeti_recalc_seeds.restype = None
        L.orc_exact_leaf_delta.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_double, C.c_double]
        L.orc_exact_leaf_delta.restype = C.c_double
        L.orc_train.argtypes = [P(_TrainArgs), P(_TrainOut)]
        L.orc_train.restype = C.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


class TFastRng64:
    """Host replica of the reference TFastRng64 (crates/cb-core/src/rng.rs)."""

    def __init__(self, seed: int | None = None, *, raw=None):
        self.s = Rng()
        if raw is not None:
            self.s.x1, self.s.c1, self.s.x2, self.s.c2 = raw
        elif seed is not None:
            lib().orc_rng_from_seed(C.byref(self.s), C.c_uint64(seed & (2**64 - 1)))

    @classmethod
    def new(cls, seed1, seq1, seed2, seq2):
        r = cls()
        lib().orc_rng_new(C.byref(r.s), seed1, seq1, seed2, seq2)
        return r

    def gen_rand(self) -> int:
        return lib().orc_rng_gen(C.byref(self.s))

    def gen_rand_real1(self) -> float:
        return lib().orc_rng_real1(C.byref(self.s))

    def advance(self, delta: int) -> None:
        lib().orc_rng_advance(C.byref(self.s), delta)

    def uniform(self, bound: int) -> int:
        return lib().orc_rng_uniform(C.byref(self.s), bound)

    def std_normal(self) -> float:
        return lib().orc_std_normal(C.byref(self.s))

    def raw_state(self):
        return (self.s.x1, self.s.c1, self.s.x2, self.s.c2)

    @property
    def call_count(self) -> int:
        return self.s.calls


def fast_logf(x: float) -> float:
    return lib().orc_fast_logf(x)


def sum_f64(v) -> float:
    v = np.ascontiguousarray(v, dtype=np.float64)
    return lib().orc_sum_f64(_p(v), v.size)


def flatten_borders(borders):
    counts = np.array([len(b) for b in borders], dtype=np.int32)
    flat = np.ascontiguousarray(np.concatenate([np.asarray(b, dtype=np.float64) for b in borders])
                                if len(borders) and counts.sum() else np.zeros(0), dtype=np.float64)
    return flat, counts


def quantize(cols_fm: np.ndarray, borders) -> np.ndarray:
    """bin_of for every (feature, object): cols_fm is f32 [F][n]."""
    cols = np.ascontiguousarray(cols_fm, dtype=np.float32)
    F, n = cols.shape
    flat, counts = flatten_borders(borders)
    out = np.empty((F, n), dtype=np.uint8)
    lib().orc_quantize(_p(cols), n, F, _p(flat), _p(counts), _p(out))
    return out


def select_borders(column, border_count: int, border_type: str = "GreedyLogSum",
                   nan_mode: str = "Min") -> np.ndarray:
    """Borders of one f32 column as the reference's builder derives them
    (builder.rs:1677-1720, border_types.rs:134-236); ascending f64."""
    col = np.ascontiguousarray(column, dtype=np.float32)
    out = np.empty(int(border_count) + 2, dtype=np.float64)
    k = lib().orc_select_borders(_p(col), col.size, int(border_count), BORDER_TYPE[border_type],
                                 NAN_MODE[nan_mode], _p(out), out.size)
    if k < 0:
        raise ValueError(f"select_borders({border_type}, nan_mode={nan_mode}) failed: {k}")
    return out[:k].copy()


def flatten_oblivious(split_feature, split_border, leaf_values):
    """CSR lowering of an oblivious ensemble (crates/cb-model/src/gpu_apply.rs:120-193):
    split_feature [T, D] (-1 = no split at that level), split_border [T, D] border
    values, leaf_values [T, 2^D] (learning-rate scaled; a tree with d splits uses
    its first 2^d values)."""
    sf = np.asarray(split_feature)
    sb = np.asarray(split_border, dtype=np.float64)
    lv = np.asarray(leaf_values, dtype=np.float64)
    feats, bords, leaves, so, lo = [], [], [], [0], [0]
    for t in range(sf.shape[0]):
        d = int(np.sum(sf[t] >= 0))
        feats.extend(int(f) for f in sf[t, :d])
        bords.extend(float(b) for b in sb[t, :d])
        leaves.extend(lv[t, : 1 << d])
        so.append(len(feats))
        lo.append(len(leaves))
    return (np.array(feats, dtype=np.uint32), np.array(bords, dtype=np.float64), np.array(so, dtype=np.uint32),
            np.array(leaves, dtype=np.float64), np.array(lo, dtype=np.uint32))


def apply_oblivious(X_fm, flat, bias=0.0, nan_above=None) -> np.ndarray:
    """Raw predictions of a flattened ensemble (crates/cb-model/src/apply.rs:374-410)."""
    x = np.ascontiguousarray(X_fm, dtype=np.float32)
    F, n = x.shape
    feats, bords, so, leaves, lo = flat
    na = None if nan_above is None else np.ascontiguousarray(nan_above, dtype=np.uint8)
    out = np.empty(n, dtype=np.float64)
    lib().orc_apply_oblivious(_p(x), n, F, _p(feats), _p(bords), _p(so), so.size - 1, _p(leaves), _p(lo),
                              float(bias), _p(na), _p(out))
    return out


def border_sample_indices(n: int, sample_size: int = 200_000) -> np.ndarray:
    """The fixed-seed sorted object sample of borders.rs:504-520."""
    m = C.c_int64(0)
    ptr = lib().orc_border_sample_indices(n, sample_size, C.byref(m))
    if not ptr:
        raise MemoryError("orc_border_sample_indices")
    arr = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_int64)), shape=(m.value,)).copy()
    C.CDLL(None).free(C.c_void_p(ptr))
    return arr


def compute_gradients(loss: str, approx, target):
    a = np.ascontiguousarray(approx, dtype=np.float64)
    t = np.ascontiguousarray(target, dtype=np.float64)
    d1 = np.empty_like(a)
    d2 = np.empty_like(a)
    lib().orc_compute_gradients(LOSS[loss], _p(a), _p(t), a.size, _p(d1), _p(d2))
    return d1, d2


def bootstrap(kind: str, der_obj, rng: TFastRng64, subsample=1.0, bagging_temperature=1.0,
              prev_leaf_mean=None):
    d = np.ascontiguousarray(der_obj, dtype=np.float64)
    sw = np.empty_like(d)
    ctl = np.empty(d.size, dtype=np.uint8)
    rc = lib().orc_bootstrap(BOOT[kind], _p(d), d.size, subsample, bagging_temperature,
                             0 if prev_leaf_mean is None else 1,
                             0.0 if prev_leaf_mean is None else prev_leaf_mean,
                             C.byref(rng.s), _p(sw), _p(ctl))
    if rc != 0:
        raise ValueError(f"bootstrap {kind} failed")
    return sw, ctl.astype(bool)


def build_histogram(bins_fm, g, h, leaf_of=None, n_leaves=1, n_bins=None):
    bins = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    F, n = bins.shape
    nb = int(n_bins if n_bins is not None else (int(bins.max()) + 1 if bins.size else 1))
    g = np.ascontiguousarray(g, dtype=np.float64)
    h = np.ascontiguousarray(h, dtype=np.float64)
    lo = None if leaf_of is None else np.ascontiguousarray(leaf_of, dtype=np.int32)
    out = np.empty((n_leaves, F, nb, 2), dtype=np.float64)
    lib().orc_build_histogram(_p(bins), n, F, nb, _p(g), _p(h), _p(lo), n_leaves, _p(out))
    return out


@dataclass
class OracleFit:
    split_feature: np.ndarray  # [iters, depth]
    split_bin: np.ndarray      # [iters, depth]
    tree_depth: np.ndarray     # [iters]
    leaf_values: np.ndarray    # [iters, 2^depth] (learning-rate scaled)
    staged: np.ndarray | None  # [iters, n]
    final_approx: np.ndarray
    bias: float
    rng_calls: np.ndarray
    level_top2: np.ndarray     # [iters, depth, 2] best and runner-up raw candidate score per level


def train(bins_fm, border_counts, target, *, loss="RMSE", depth=6, iterations=10,
          learning_rate=0.1, l2_leaf_reg=3.0, score_function="Cosine", bootstrap_type="No",
          subsample=0.66, bagging_temperature=1.0, random_strength=0.0, random_seed=0,
          boost_from_average=True, weights=None, staged=True, n_threads=0, cat_bins_fm=None,
          leaf_estimation_method="Gradient", quantile_alpha=0.5, quantile_delta=1e-6) -> OracleFit:
    """The reference CPU boosting loop (crates/cb-train/src/boosting.rs) on quantized bins;
    cat_bins_fm [C, n] adds one-hot categorical features (split_feature >= F: cat feature
    split_feature - F, passing on bin == split_bin).  leaf_estimation_method "Exact" takes
    each leaf's weighted quantile of the residuals (MAE / Quantile only, boosting.rs:2561-2606);
    quantile_alpha / quantile_delta are Quantile's parameters (MAE is alpha 0.5, delta 1e-6)."""
    if leaf_estimation_method not in ("Gradient", "Exact"):
        raise ValueError(f"leaf method {leaf_estimation_method} is not restated")
    exact = leaf_estimation_method == "Exact"
    if exact and loss not in ("MAE", "Quantile"):
        raise ValueError("the Exact leaf is restated for MAE and Quantile")
    bins = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    F, n = bins.shape
    cb = None if cat_bins_fm is None else np.ascontiguousarray(cat_bins_fm, dtype=np.uint8).reshape(-1, n)
    bc = np.ascontiguousarray(border_counts, dtype=np.int32)
    t = np.ascontiguousarray(target, dtype=np.float64)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    L = 1 << depth
    sf = np.empty((iterations, depth), dtype=np.int32)
    sb = np.empty((iterations, depth), dtype=np.int32)
    td = np.empty(iterations, dtype=np.int32)
    lv = np.empty((iterations, L), dtype=np.float64)
    st = np.empty((iterations, n), dtype=np.float64) if staged else None
    fa = np.empty(n, dtype=np.float64)
    bias = np.zeros(1, dtype=np.float64)
    calls = np.zeros(iterations, dtype=np.uint64)
    top2 = np.full((iterations, depth, 2), -np.inf, dtype=np.float64)
    args = _TrainArgs(n, F, _p(bins), _p(bc), _p(t), _p(w), LOSS[loss], depth, iterations,
                      learning_rate, l2_leaf_reg, SCORE[score_function], BOOT[bootstrap_type],
                      subsample, bagging_temperature, random_strength, random_seed,
                      1 if boost_from_average else 0, n_threads, 0 if cb is None else cb.shape[0], _p(cb),
                      1 if exact else 0, quantile_alpha, quantile_delta)
    out = _TrainOut(_p(sf), _p(sb), _p(td), _p(lv), _p(st), _p(fa), _p(bias), _p(calls), _p(top2))
    rc = lib().orc_train(C.byref(args), C.byref(out))
    if rc != 0:
        raise RuntimeError(f"orc_train failed rc={rc}")
    return OracleFit(sf, sb, td, lv, st, fa, float(bias[0]), calls, top2)


@dataclass
class OracleMultiFit:
    split_feature: np.ndarray  # [iters, depth]
    split_bin: np.ndarray      # [iters, depth]
    tree_depth: np.ndarray     # [iters]
    leaf_values: np.ndarray    # [iters, 2^depth, K] (leaf-major, learning-rate scaled)
    staged: np.ndarray | None  # [iters, n, K]
    final_approx: np.ndarray   # [n, K]


MULTI_LOSSES = ("MultiClass", "MultiClassOneVsAll", "MultiLogloss", "MultiCrossEntropy", "RMSEWithUncertainty")


def train_multiclass(bins_fm, border_counts, target_class, n_classes, *, depth=6, iterations=10,
                     learning_rate=0.1, l2_leaf_reg=3.0, score_function="Cosine", bootstrap_type="No",
                     subsample=0.66, bagging_temperature=1.0, random_seed=0, weights=None, staged=True,
                     n_threads=0, cat_bins_fm=None, loss="MultiClass") -> OracleMultiFit:
    """The reference's multi-output CPU loop on quantized bins, Newton leaves.

    loss "MultiClass" (softmax, dense Hessian solve) and "MultiClassOneVsAll"
    take class indices in target_class; "MultiLogloss" and "MultiCrossEntropy"
    take a [K, n] label matrix (dim-major), all three diagonal losses solving
    each dimension on its own (boosting.rs:8323-8420).  cat_bins_fm [C, n] adds
    one-hot categorical features (split_feature >= F)."""
    bins = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    F, n = bins.shape
    cb = None if cat_bins_fm is None else np.ascontiguousarray(cat_bins_fm, dtype=np.uint8).reshape(-1, n)
    K = int(n_classes)
    bc = np.ascontiguousarray(border_counts, dtype=np.int32)
    if loss not in MULTI_LOSSES:
        raise ValueError(f"unknown multi-output loss {loss}")
    tm = None
    if loss == "MultiClass":
        y = np.ascontiguousarray(target_class, dtype=np.int32)
    elif loss == "MultiClassOneVsAll":
        y = np.ascontiguousarray(target_class, dtype=np.int32)
        tm = np.ascontiguousarray((np.arange(K)[:, None] == y[None, :]).astype(np.float64))
    elif loss == "RMSEWithUncertainty":
        if K != 2:
            raise ValueError("RMSEWithUncertainty has two dimensions")
        tm = np.ascontiguousarray(target_class, dtype=np.float64).reshape(n)
        y = None
    else:
        tm = np.ascontiguousarray(target_class, dtype=np.float64).reshape(K, n)
        y = None
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    L = 1 << depth
    sf = np.empty((iterations, depth), dtype=np.int32)
    sb = np.empty((iterations, depth), dtype=np.int32)
    td = np.empty(iterations, dtype=np.int32)
    lv = np.empty((iterations, L, K), dtype=np.float64)
    st = np.empty((iterations, n, K), dtype=np.float64) if staged else None
    fa = np.empty((n, K), dtype=np.float64)
    args = _MultiArgs(n, F, _p(bins), _p(bc), _p(y), _p(w), K, depth, iterations, learning_rate, l2_leaf_reg,
                      SCORE[score_function], BOOT[bootstrap_type], subsample, bagging_temperature, random_seed,
                      n_threads, 0 if cb is None else cb.shape[0], _p(cb), 0 if tm is None else (2 if loss == "RMSEWithUncertainty" else 1), _p(tm))
    out = _MultiOut(_p(sf), _p(sb), _p(td), _p(lv), _p(st), _p(fa))
    rc = lib().orc_train_multiclass(C.byref(args), C.byref(out))
    if rc != 0:
        raise RuntimeError(f"orc_train_multiclass failed rc={rc}")
    return OracleMultiFit(sf, sb, td, lv, st, fa)


def exact_leaf_delta(residuals, weights, alpha=0.5, delta=1e-6) -> float:
    r = np.ascontiguousarray(residuals, dtype=np.float32)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    return lib().orc_exact_leaf_delta(_p(r), _p(w), r.size, alpha, delta)


def solve_symmetric_newton(sum_der, sum_der2_packed, scaled_l2):
    d = np.ascontiguousarray(sum_der, dtype=np.float64)
    h = np.ascontiguousarray(sum_der2_packed, dtype=np.float64)
    out = np.empty(d.size, dtype=np.float64)
    lib().orc_solve_symmetric_newton(_p(d), _p(h), d.size, scaled_l2, _p(out))
    return out


@dataclass
class OracleRankFit:
    split_feature: np.ndarray   # [iters, depth]
    split_bin: np.ndarray       # [iters, depth]
    leaf_values: np.ndarray     # [iters, 2^depth] normalised and learning-rate scaled
    raw_leaf_values: np.ndarray  # [iters, 2^depth] Newton deltas
    staged: np.ndarray | None   # [iters, n]


def train_ranking(bins_fm, border_counts, target, group_offsets, *, loss="QueryRMSE", pairs=None, depth=6,
                  iterations=10, learning_rate=0.1, l2_leaf_reg=3.0, score_function="Cosine", random_seed=0,
                  weights=None, staged=True, softmax_lambda=0.01, softmax_beta=1.0, lambdamart_sigma=1.0,
                  lambdamart_top=-1, lambdamart_norm=True, yeti_permutations=10,
                  yeti_decay=0.85, srank_metric="DCG", srank_sigma=1.0, srank_mu=0.0,
                  srank_num_estimations=1, lambdamart_metric="NDCG", pair_weights=None) -> OracleRankFit:
    """The reference's grouped-loss CPU loop: QueryRMSE / PairLogit (pointwise histograms, Newton
    leaves), QuerySoftMax (pointwise histograms, Gradient leaves), LambdaMart (NDCG lambdas, Newton
    leaves), YetiRank (sampled pairs, Newton leaves, two approximants), StochasticRank (Monte-Carlo
    DCG / NDCG ders, Gradient leaves) and PairLogitPairwise (pairwise scoring, Cholesky pairwise
    leaves)."""
    bins = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    F, n = bins.shape
    bc = np.ascontiguousarray(border_counts, dtype=np.int32)
    t = np.ascontiguousarray(target, dtype=np.float64)
    go = np.ascontiguousarray(group_offsets, dtype=np.int64)
    pr = np.zeros((0, 2), dtype=np.int64) if pairs is None else np.ascontiguousarray(pairs, dtype=np.int64)
    pw = np.ascontiguousarray(pr[:, 0])
    pl = np.ascontiguousarray(pr[:, 1])
    pwt = None if pair_weights is None else np.ascontiguousarray(pair_weights, dtype=np.float64)
    if pwt is not None and pwt.size != pw.size:
        raise ValueError("pair_weights must have one weight per pair")
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    L = 1 << depth
    sf = np.empty((iterations, depth), dtype=np.int32)
    sb = np.empty((iterations, depth), dtype=np.int32)
    lv = np.empty((iterations, L), dtype=np.float64)
    raw = np.empty((iterations, L), dtype=np.float64)
    st = np.empty((iterations, n), dtype=np.float64) if staged else None
    args = _RankArgs(n, F, _p(bins), _p(bc), _p(t), _p(w), RANK_LOSS[loss], go.size - 1, _p(go), pw.size, _p(pw),
                     _p(pl), depth, iterations, learning_rate, l2_leaf_reg, SCORE[score_function], random_seed,
                     softmax_lambda, softmax_beta, lambdamart_sigma, lambdamart_top, int(bool(lambdamart_norm)),
                     yeti_permutations, yeti_decay, 1 if srank_metric == "NDCG" else 0, srank_sigma, srank_mu,
                     srank_num_estimations, 1 if lambdamart_metric in ("MRR", "ERR", "MAP") else 0, _p(pwt))
    out = _RankOut(_p(sf), _p(sb), _p(lv), _p(raw), _p(st))
    rc = lib().orc_train_ranking(C.byref(args), C.byref(out))
    if rc != 0:
        raise RuntimeError(f"orc_train_ranking failed rc={rc}")
    return OracleRankFit(sf, sb, lv, raw, st)


def yeti_sample_pairs(raw_approx, relevs, query_weight=1.0, permutations=10, decay=0.85, query_seed=0):
    """YetiRank's per-group pair sampler (crates/cb-train/src/yetirank.rs:75-171): the dense
    [g, g] matrix of sampled pair weights, winner row over loser column."""
    a = np.ascontiguousarray(raw_approx, dtype=np.float64)
    r = np.ascontiguousarray(relevs, dtype=np.float64)
    out = np.zeros((a.size, a.size), dtype=np.float64)
    lib().orc_yeti_sample_pairs(_p(a), _p(r), a.size, query_weight, permutations, decay,
                                C.c_uint64(query_seed & (2**64 - 1)), _p(out))
    return out


def yeti_query_seeds(random_seed: int, n_groups: int) -> np.ndarray:
    out = np.zeros(n_groups, dtype=np.uint64)
    lib().orc_yeti_query_seeds(C.c_uint64(random_seed), n_groups, _p(out))
    return out


def yeti_recalc_seeds(random_seed: int, n_groups: int, n_features: int, depth: int, trees: int) -> np.ndarray:
    """The per-tree (deriv, learning-fold, leaf-value) recalc seeds of YetiRankTreeSeeder."""
    out = np.zeros((trees, 3), dtype=np.uint64)
    lib().orc_yeti_recalc_seeds(C.c_uint64(random_seed), n_groups, n_features, depth, trees, _p(out))
    return out


def city_hash64(s: str) -> int:
    """CityHash64 v1.0 of the UTF-8 string."""
    b = s.encode()
    return lib().orc_city_hash64(b, len(b))


def cat_hash(s: str) -> int:
    """CalcCatFeatureHash: the low 32 bits of CityHash64 of the category's string form."""
    b = s.encode()
    return lib().orc_cat_hash(b, len(b))


def perfect_hash_bins(values) -> tuple:
    """The perfect-hash bins of one categorical column: bin = first-seen order.  Returns
    (bins [n] uint8/uint32, the distinct values in bin order)."""
    index = {}
    out = np.empty(len(values), dtype=np.uint32)
    for i, v in enumerate(values):
        out[i] = index.setdefault(v, len(index))
    return out, list(index)


def score_term(score_function: str, sum_der: float, weight: float) -> float:
    """One leaf's SolarL2 / LOOL2 / SatL2 score term (score.rs:266-330)."""
    return lib().orc_score_term(SCORE[score_function], sum_der, weight)
