"""Host-side mirror of the reference's device seam, `cb_compute::Runtime`
(crates/cb-compute/src/runtime.rs:1410-1651), backed by libcbgpu.so.

Method names, argument meaning and decline/error behaviour follow the trait:
begin_* returns False when the session declines (the trait's Ok(false)),
grow_tree_on_device returns None when no session is open (Ok(None)), and
invalid input raises CbGpuError (the CbError analogue: LengthMismatch /
Degenerate).  The types mirror DeviceTrainConfig (runtime.rs:1259-1372) and
DeviceGrownTree (runtime.rs:989-1059).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _lib

LOSS = {"RMSE": 0, "Rmse": 0, "Logloss": 1, "CrossEntropy": 2, "MultiClass": 3, "QueryRMSE": 4, "PairLogit": 5,
        "PairLogitPairwise": 6, "QuerySoftMax": 7,
        "LambdaMart": 8, "YetiRank": 9, "StochasticRank": 10, "YetiRankPairwise": 11, "MultiClassOneVsAll": 12,
        "MultiLogloss": 13, "MultiCrossEntropy": 14, "MAE": 15, "Quantile": 16,
        "RMSEWithUncertainty": 17}
# multi-output losses whose target is the [K, n] label matrix (dim-major)
LABEL_MATRIX_LOSSES = ("MultiLogloss", "MultiCrossEntropy")
LAMBDAMART_METRIC = {"NDCG": 0, "DCG": 1, "MRR": 2, "ERR": 3, "MAP": 4}
SCORE = {"Cosine": 0, "L2": 1, "SolarL2": 2, "NewtonL2": 3, "NewtonCosine": 4, "LOOL2": 5, "SatL2": 6}
BOOT = {"No": 0, "Bayesian": 1, "Bernoulli": 2, "MVS": 3, "Mvs": 3, "Poisson": 4}
GROW = {"SymmetricTree": 0, "Depthwise": 1, "Lossguide": 2, "Region": 3}
BORDER_TYPE = {"Median": 0, "GreedyLogSum": 1, "UniformAndQuantiles": 2, "MinEntropy": 3,
               "MaxLogSum": 4, "Uniform": 5, "GreedyMinEntropy": 6}
NAN_MODE = {"Min": 0, "Max": 1, "Forbidden": 2}


@dataclass
class DeviceTrainConfig:
    """DeviceTrainConfig (runtime.rs:1259-1372) plus this build's placement fields."""
    grow_policy: str = "SymmetricTree"
    bootstrap_type: str = "No"
    sample_rate: float = 1.0
    mvs_lambda: Optional[float] = None
    rng_seed: int = 0
    bias: float = 0.0
    sample_from_host: bool = False
    bagging_temperature: float = 1.0
    random_strength: float = 0.0
    border_counts: Optional[Sequence[int]] = None
    # Exact leaves for MAE / Quantile (DeviceTrainConfig::exact_leaf, quantile_alpha / _delta)
    exact_leaf: bool = False
    quantile_alpha: float = 0.5
    quantile_delta: float = 1e-6
    # document sharding (one process per GPU)
    device: int = 0
    rank: int = 0
    world_size: int = 1
    row_offset: int = 0
    n_total: Optional[int] = None
    nccl_unique_id: Optional[bytes] = None


@dataclass
class Derivatives:
    der1: np.ndarray
    der2: np.ndarray


@dataclass
class DeviceGrownTree:
    """DeviceGrownTree (runtime.rs:989-1059) for the oblivious arm."""
    splits: list                  # [(feature, bin_id, is_one_hot)] in level order (bit l = split l)
    leaf_values: np.ndarray       # 2^depth raw deltas, NOT scaled by learning_rate
    approx_dim: int = 1
    leaf_of: np.ndarray = field(default_factory=lambda: np.zeros(0, dtype=np.uint32))
    step_nodes: list = field(default_factory=list)
    node_id_to_leaf_id: list = field(default_factory=list)
    region_path: list = field(default_factory=list)


def _ptr(a):
    return None if a is None else a.ctypes.data


def nccl_unique_id() -> bytes:
    L = _lib.load()
    buf = (C.c_uint8 * 128)()
    _lib.check(L.cbgpu_nccl_unique_id(buf))
    return bytes(buf)


class B200Runtime:
    """`impl Runtime` for the B200 backend (one session per fit)."""

    def __init__(self):
        self._L = _lib.load()
        self._s = C.c_void_p(None)
        self._staged = []  # host samples whose uploads (cbgpu_stage_sample) wait for their trees
        self.n = 0
        self.depth = 0
        self.decline_reason = ""
        self._keep = []

    # ---- Runtime::compute_gradients (runtime.rs:1431) -----------------------
    def compute_gradients(self, loss, approx, target, approx_dimension: int = 1) -> Derivatives:
        if approx_dimension != 1:
            raise _lib.CbGpuError(_lib.DECLINED, "approx_dimension != 1 is not covered")
        a = np.ascontiguousarray(approx, dtype=np.float64)
        t = np.ascontiguousarray(target, dtype=np.float64)
        if a.shape != t.shape:
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: approx vs target")
        d1, d2 = np.empty_like(a), np.empty_like(a)
        rc = self._L.cbgpu_compute_gradients(LOSS[loss], _ptr(a), _ptr(t), a.size, _ptr(d1), _ptr(d2))
        if rc == _lib.DECLINED:
            raise _lib.CbGpuError(rc, _lib.last_error())
        _lib.check(rc)
        return Derivatives(d1, d2)

    # ---- begin -------------------------------------------------------------
    def _args(self, loss, depth, plain, fold_count, score_function, weight, n, n_features, n_bins,
              learning_rate, scaled_l2, cfg: DeviceTrainConfig):
        w = None if weight is None or len(weight) == 0 else np.ascontiguousarray(weight, dtype=np.float64)
        if w is not None and w.size != n:
            raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: weight has {w.size}, expected {n}")
        bc = None if cfg.border_counts is None else np.ascontiguousarray(cfg.border_counts, dtype=np.int32)
        uid = None
        if cfg.world_size > 1:
            if cfg.nccl_unique_id is None or len(cfg.nccl_unique_id) != 128:
                raise _lib.CbGpuError(_lib.ERR_INVALID, "world_size > 1 needs a 128-byte nccl_unique_id")
            uid = np.frombuffer(cfg.nccl_unique_id, dtype=np.uint8).copy()
        self._keep = [w, bc, uid]
        a = _lib.BeginArgs()
        a.loss = LOSS[loss]
        a.depth = depth
        a.boosting_type_is_plain = 1 if plain else 0
        a.fold_count = fold_count
        a.score_function = SCORE[score_function]
        a.n = n
        a.n_features = n_features
        a.n_bins = n_bins
        a.learning_rate = learning_rate
        a.scaled_l2 = scaled_l2
        a.weight = _ptr(w)
        a.grow_policy = GROW[cfg.grow_policy]
        a.bootstrap_type = BOOT[cfg.bootstrap_type]
        a.sample_rate = cfg.sample_rate
        a.bagging_temperature = cfg.bagging_temperature
        a.has_mvs_lambda = 0 if cfg.mvs_lambda is None else 1
        a.mvs_lambda = 0.0 if cfg.mvs_lambda is None else cfg.mvs_lambda
        a.rng_seed = cfg.rng_seed & (2**64 - 1)
        a.bias = cfg.bias
        a.sample_from_host = 1 if cfg.sample_from_host else 0
        a.random_strength = cfg.random_strength
        a.device = cfg.device
        a.rank = cfg.rank
        a.world_size = cfg.world_size
        a.row_offset = cfg.row_offset
        a.n_total = cfg.n_total if cfg.n_total is not None else n
        a.nccl_unique_id = _ptr(uid)
        a.border_counts = _ptr(bc)
        a.exact_leaf = 1 if cfg.exact_leaf else 0
        a.quantile_alpha = cfg.quantile_alpha
        a.quantile_delta = cfg.quantile_delta
        return a

    def _finish_begin(self, rc, n, depth) -> bool:
        if rc == _lib.DECLINED:
            self.decline_reason = _lib.last_error()
            self._s = C.c_void_p(None)
            return False
        _lib.check(rc)
        self.n, self.depth = n, depth
        return True

    def begin_device_training(self, loss, depth, boosting_type_is_plain, fold_count, score_function,
                              bins_feature_major, weight, n, n_features, n_bins, learning_rate,
                              scaled_l2, config: DeviceTrainConfig) -> bool:
        """Runtime::begin_device_training (runtime.rs:1497): u32 feature-major bins."""
        self.end_device_training()
        bins = np.ascontiguousarray(bins_feature_major, dtype=np.uint32).reshape(-1)
        if bins.size != n * n_features:
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: bins_feature_major")
        a = self._args(loss, depth, boosting_type_is_plain, fold_count, score_function, weight, n,
                       n_features, n_bins, learning_rate, scaled_l2, config)
        rc = self._L.cbgpu_begin(C.byref(a), _ptr(bins), C.byref(self._s))
        return self._finish_begin(rc, n, depth)

    def begin_device_training_raw(self, loss, depth, boosting_type_is_plain, fold_count, score_function,
                                  float_columns, feature_borders, weight, n, n_features, n_bins,
                                  learning_rate, scaled_l2, config: DeviceTrainConfig) -> bool:
        """Runtime::begin_device_training_raw (runtime.rs:1546): device quantization."""
        self.end_device_training()
        cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
        if len(cols) != n_features or any(c.size != n for c in cols):
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: float_columns")
        counts = np.array([len(b) for b in feature_borders], dtype=np.int32)
        flat = np.ascontiguousarray(
            np.concatenate([np.asarray(b, dtype=np.float64) for b in feature_borders])
            if counts.sum() else np.zeros(1), dtype=np.float64)
        colptrs = (C.c_void_p * max(1, len(cols)))(*[c.ctypes.data for c in cols])
        a = self._args(loss, depth, boosting_type_is_plain, fold_count, score_function, weight, n,
                       n_features, n_bins, learning_rate, scaled_l2, config)
        rc = self._L.cbgpu_begin_raw(C.byref(a), colptrs, _ptr(flat), _ptr(counts), C.byref(self._s))
        return self._finish_begin(rc, n, depth)

    # ---- Runtime::grow_tree_on_device (runtime.rs:1629) ---------------------
    def grow_tree_on_device(self, approx, target, sample, family=None, leaf_of_bytes: int = 4,
                            resident_approx: bool = False) -> Optional[DeviceGrownTree]:
        if not self._s:
            return None
        if family is not None:
            raise _lib.CbGpuError(_lib.DECLINED, "family trees (ranking/pairwise/multi-output) are not covered")
        a = None if resident_approx or approx is None else np.ascontiguousarray(approx, dtype=np.float64)
        t = None if target is None else np.ascontiguousarray(target, dtype=np.float64)
        s = None if sample is None or len(sample) == 0 else np.ascontiguousarray(sample, dtype=np.float64)
        if a is not None and a.size != self.n:
            raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: approx has {a.size}, expected {self.n}")
        if t is not None and t.size != self.n:
            raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: target has {t.size}, expected {self.n}")
        D = self.depth
        sf = np.empty(D, dtype=np.int32)
        sb = np.empty(D, dtype=np.int32)
        ns = np.zeros(1, dtype=np.int32)
        lv = np.empty(1 << D, dtype=np.float64)
        lo = None
        if leaf_of_bytes:
            lo = np.empty(self.n, dtype={1: np.uint8, 2: np.uint16, 4: np.uint32}[leaf_of_bytes])
        rc = self._L.cbgpu_grow_tree(self._s, _ptr(a), _ptr(t), self.n, _ptr(s),
                                     0 if s is None else s.size, _ptr(sf), _ptr(sb), _ptr(ns), _ptr(lv),
                                     _ptr(lo), leaf_of_bytes if lo is not None else 0)
        if rc == 0 and s is None and self._staged:
            self._staged.pop(0)  # the tree took (and finished with) the oldest staged sample
        _lib.check(rc)
        k = int(ns[0])
        return DeviceGrownTree(splits=[(int(sf[i]), int(sb[i]), False) for i in range(k)],
                               leaf_values=lv,
                               leaf_of=lo if lo is not None else np.zeros(0, dtype=np.uint32))

    def stage_sample(self, sample) -> None:
        """Start uploading the host bootstrap sample of a later grow call
        (cbgpu_stage_sample): a grow_tree_on_device call with no sample takes
        the oldest staged one, so staging tree t + 1's sample before growing
        tree t overlaps its upload with tree t's device work.  The array is
        kept alive here until its tree has grown; pinned memory overlaps."""
        if not self._s:
            raise _lib.CbGpuError(_lib.ERR_INVALID, "no session")
        arr = sample if (isinstance(sample, np.ndarray) and sample.dtype == np.float64
                         and sample.flags.c_contiguous) else np.ascontiguousarray(sample, dtype=np.float64)
        _lib.check(self._L.cbgpu_stage_sample(self._s, _ptr(arr), arr.size))
        self._staged.append(arr)

    def end_device_training(self) -> None:
        if self._s:
            self._L.cbgpu_end(self._s)
            self._s = C.c_void_p(None)
        self._staged = []

    def __del__(self):
        try:
            self.end_device_training()
        except Exception:
            pass

    # ---- session introspection ---------------------------------------------
    def resident_approx(self) -> np.ndarray:
        out = np.empty(self.n, dtype=np.float64)
        _lib.check(self._L.cbgpu_session_approx(self._s, _ptr(out), self.n))
        return out

    def device_bins(self, n_features: int) -> np.ndarray:
        out = np.empty((n_features, self.n), dtype=np.uint8)
        _lib.check(self._L.cbgpu_session_bins(self._s, _ptr(out), self.n, n_features))
        return out

    def last_sample(self) -> np.ndarray:
        out = np.empty(self.n, dtype=np.float64)
        _lib.check(self._L.cbgpu_session_last_sample(self._s, _ptr(out), self.n))
        return out

    def set_profiling(self, on: bool) -> None:
        _lib.check(self._L.cbgpu_session_set_profiling(self._s, 1 if on else 0))

    def set_graphs(self, on: bool) -> None:
        """Replay each tree as one captured CUDA graph (default) or enqueue it."""
        _lib.check(self._L.cbgpu_session_set_graphs(self._s, 1 if on else 0))

    def timing(self) -> np.ndarray:
        """[tree ms, hist ms, derive+score ms, partition ms, der+bootstrap ms,
        collectives ms, rows histogrammed, kernels launched] of the last tree."""
        out = np.zeros(8, dtype=np.float64)
        _lib.check(self._L.cbgpu_session_timing(self._s, _ptr(out)))
        return out

    def timing_sum(self, reset: bool = False) -> np.ndarray:
        """The timing() figures summed over the trees since the last reset."""
        out = np.zeros(8, dtype=np.float64)
        _lib.check(self._L.cbgpu_session_timing_sum(self._s, _ptr(out), 1 if reset else 0))
        return out

    def mark(self, slot: int) -> None:
        """Record user event `slot` (0..3) on the session stream."""
        _lib.check(self._L.cbgpu_session_mark(self._s, slot))

    def elapsed_ms(self, a: int, b: int) -> float:
        out = np.zeros(1, dtype=np.float64)
        _lib.check(self._L.cbgpu_session_elapsed_ms(self._s, a, b, _ptr(out)))
        return float(out[0])

    def rng_state(self):
        out = np.zeros(5, dtype=np.uint64)
        _lib.check(self._L.cbgpu_session_rng_state(self._s, _ptr(out)))
        return tuple(int(x) for x in out[:4]), int(out[4])


class B200MultiRuntime(B200Runtime):
    """The seam's multi-output family (FamilyTreeArgs::MultiOutput,
    runtime.rs:935-948) for MultiClass: the same method names as the scalar
    runtime, with a K-dimensional approximant (dim-major, approx_k[d * n + i])
    and leaf_count x K leaf blocks.  Backed by cbgpu_multi_* (one GPU)."""

    def __init__(self):
        super().__init__()
        self.approx_dim = 0
        self.label_matrix = False

    def begin_device_training_raw(self, loss, depth, boosting_type_is_plain, fold_count, score_function,
                                  float_columns, feature_borders, weight, n, n_features, n_bins,
                                  learning_rate, scaled_l2, config: DeviceTrainConfig, approx_dim: int = 2,
                                  cat_columns=None) -> bool:
        """The multi-output arm's begin; cat_columns are one-hot categorical
        features as perfect-hash bins (first-seen order, uint32 per object),
        split features n_features + c."""
        self.end_device_training()
        cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
        if len(cols) != n_features or any(c.size != n for c in cols):
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: float_columns")
        counts = np.array([len(b) for b in feature_borders], dtype=np.int32)
        flat = np.ascontiguousarray(
            np.concatenate([np.asarray(b, dtype=np.float64) for b in feature_borders])
            if counts.sum() else np.zeros(1), dtype=np.float64)
        colptrs = (C.c_void_p * max(1, len(cols)))(*[c.ctypes.data for c in cols])
        a = self._args(loss, depth, boosting_type_is_plain, fold_count, score_function, weight, n,
                       n_features, n_bins, learning_rate, scaled_l2, config)
        cats = [np.ascontiguousarray(c, dtype=np.uint32) for c in (cat_columns or [])]
        if any(c.size != n for c in cats):
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: cat_columns")
        catptrs = (C.c_void_p * max(1, len(cats)))(*[c.ctypes.data for c in cats])
        self._keep += cats
        rc = self._L.cbgpu_multi_begin_cat_raw(C.byref(a), int(approx_dim), colptrs, _ptr(flat), _ptr(counts),
                                               len(cats), catptrs, C.byref(self._s))
        ok = self._finish_begin(rc, n, depth)
        self.approx_dim = int(approx_dim) if ok else 0
        self.label_matrix = ok and loss in LABEL_MATRIX_LOSSES
        return ok

    def begin_device_training(self, *args, **kwargs) -> bool:
        raise _lib.CbGpuError(_lib.DECLINED, "the multi-output arm quantizes on the device (begin_raw)")

    def begin_ranking_raw(self, loss, depth, boosting_type_is_plain, fold_count, score_function, float_columns,
                          feature_borders, weight, n, n_features, n_bins, learning_rate, scaled_l2,
                          config: DeviceTrainConfig, group_offsets, pairs=None, l2_leaf_reg=None,
                          softmax_lambda=0.01, softmax_beta=1.0, lambdamart_sigma=1.0, lambdamart_top=-1,
                          lambdamart_norm=True, lambdamart_metric="NDCG", yeti_permutations=10,
                          yeti_decay=0.85, srank_metric="DCG", srank_sigma=1.0, srank_mu=0.0,
                          srank_num_estimations=1, pair_weights=None) -> bool:
        """The grouped families (FamilyTreeArgs::Ranking / ::Pairwise) for
        QueryRMSE / QuerySoftMax / LambdaMart / YetiRank / StochasticRank / PairLogit /
        PairLogitPairwise: group offsets
        [n_groups + 1] and, for the pair losses, (winner, loser) global object
        ids with optional per-pair weights (Competitor::weight; default 1);
        l2_leaf_reg is the unscaled l2 the pairwise scorer and leaves use
        (default scaled_l2); QuerySoftMax's lambda and beta; LambdaMart's
        sigma, top, norm and metric (NDCG / DCG); YetiRank's permutations and
        decay (its pairs are sampled on the device); StochasticRank's metric
        (DCG / NDCG), sigma, mu and num_estimations; grown with
        grow_tree_on_device (family None, approx_dim 1)."""
        self.end_device_training()
        cols = [np.ascontiguousarray(c, dtype=np.float32) for c in float_columns]
        if len(cols) != n_features or any(c.size != n for c in cols):
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: float_columns")
        counts = np.array([len(b) for b in feature_borders], dtype=np.int32)
        flat = np.ascontiguousarray(
            np.concatenate([np.asarray(b, dtype=np.float64) for b in feature_borders])
            if counts.sum() else np.zeros(1), dtype=np.float64)
        colptrs = (C.c_void_p * max(1, len(cols)))(*[c.ctypes.data for c in cols])
        go = np.ascontiguousarray(group_offsets, dtype=np.int64)
        pr = np.zeros((0, 2), dtype=np.int64) if pairs is None else np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
        pw = np.ascontiguousarray(pr[:, 0])
        pl = np.ascontiguousarray(pr[:, 1])
        pwt = None if pair_weights is None else np.ascontiguousarray(pair_weights, dtype=np.float64)
        if pwt is not None and pwt.size != pw.size:
            raise _lib.CbGpuError(_lib.ERR_INVALID, "LengthMismatch: pair_weights must have one weight per pair")
        a = self._args(loss, depth, boosting_type_is_plain, fold_count, score_function, weight, n,
                       n_features, n_bins, learning_rate, scaled_l2, config)
        self._keep += [go, pw, pl] + ([pwt] if pwt is not None else [])
        rp = _lib.RankParams(-1.0 if l2_leaf_reg is None else float(l2_leaf_reg), float(softmax_lambda),
                             float(softmax_beta), float(lambdamart_sigma), int(lambdamart_top),
                             1 if lambdamart_norm else 0, LAMBDAMART_METRIC[lambdamart_metric],
                             int(yeti_permutations), float(yeti_decay), LAMBDAMART_METRIC[srank_metric],
                             int(srank_num_estimations), float(srank_sigma), float(srank_mu), _ptr(pwt))
        rc = self._L.cbgpu_rank_begin_raw(C.byref(a), _ptr(go), go.size - 1, _ptr(pw), _ptr(pl), pw.size,
                                          C.byref(rp), colptrs, _ptr(flat), _ptr(counts), C.byref(self._s))
        ok = self._finish_begin(rc, n, depth)
        self.approx_dim = 1 if ok else 0
        return ok

    def grow_tree_on_device(self, approx, target, sample, family=None, leaf_of_bytes: int = 4,
                            resident_approx: bool = False) -> Optional[DeviceGrownTree]:
        """family = ("MultiOutput", approx_k, approx_dim); approx_k None with
        resident_approx uses the session's own approximant."""
        if not self._s:
            return None
        K, n, D = self.approx_dim, self.n, self.depth
        ak = None
        if family is None and not resident_approx and approx is not None and K == 1:
            ak = np.ascontiguousarray(approx, dtype=np.float64).reshape(-1)  # the grouped families (K = 1)
            if ak.size != n:
                raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: approx has {ak.size}, expected {n}")
        if family is not None:
            kind, fam_approx, fam_dim = family
            if kind != "MultiOutput" or int(fam_dim) != K:
                raise _lib.CbGpuError(_lib.DECLINED, f"family {kind} / dim {fam_dim} not covered")
            if not resident_approx and fam_approx is not None:
                ak = np.ascontiguousarray(fam_approx, dtype=np.float64).reshape(-1)
                if ak.size != K * n:
                    raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: approx_k has {ak.size}, expected {K * n}")
        t = None if target is None else np.ascontiguousarray(target, dtype=np.float64).reshape(-1)
        s = None if sample is None or len(sample) == 0 else np.ascontiguousarray(sample, dtype=np.float64)
        want = K * n if self.label_matrix else n
        if t is not None and t.size != want:
            raise _lib.CbGpuError(_lib.ERR_INVALID, f"LengthMismatch: target has {t.size}, expected {want}")
        sf = np.empty(D, dtype=np.int32)
        sb = np.empty(D, dtype=np.int32)
        ns = np.zeros(1, dtype=np.int32)
        lv = np.empty((1 << D) * K, dtype=np.float64)
        lo = None
        if leaf_of_bytes:
            lo = np.empty(n, dtype={1: np.uint8, 2: np.uint16, 4: np.uint32}[leaf_of_bytes])
        rc = self._L.cbgpu_multi_grow_tree(self._s, _ptr(ak), _ptr(t), n, _ptr(s), 0 if s is None else s.size,
                                           _ptr(sf), _ptr(sb), _ptr(ns), _ptr(lv), _ptr(lo),
                                           leaf_of_bytes if lo is not None else 0)
        _lib.check(rc)
        k = int(ns[0])
        return DeviceGrownTree(splits=[(int(sf[i]), int(sb[i]), False) for i in range(k)], leaf_values=lv,
                               approx_dim=K, leaf_of=lo if lo is not None else np.zeros(0, dtype=np.uint32))

    def end_device_training(self) -> None:
        if self._s:
            self._L.cbgpu_multi_end(self._s)
            self._s = C.c_void_p(None)

    def resident_approx(self) -> np.ndarray:
        """The resident approximant, dim-major [K, n]."""
        out = np.empty((self.approx_dim, self.n), dtype=np.float64)
        _lib.check(self._L.cbgpu_multi_approx(self._s, _ptr(out), self.n))
        return out

    def device_bins(self, n_features):
        raise NotImplementedError("multi-output sessions do not export their bins")

    def last_sample(self):
        raise NotImplementedError("multi-output sessions do not export their sample")


# ---- building blocks -------------------------------------------------------

def histogram(bins_row_major, g, h, leaf_of=None, n_leaves=1, n_bins=None) -> np.ndarray:
    """Device level histogram, [leaf][feature][bin][2] (sum g, sum h)."""
    L = _lib.load()
    bins = np.ascontiguousarray(bins_row_major, dtype=np.uint8)
    n, F = bins.shape
    B = int(n_bins if n_bins is not None else (int(bins.max()) + 1 if bins.size else 1))
    g = np.ascontiguousarray(g, dtype=np.float64)
    h = np.ascontiguousarray(h, dtype=np.float64)
    lo = None if leaf_of is None else np.ascontiguousarray(leaf_of, dtype=np.int32)
    out = np.empty((n_leaves, F, B, 2), dtype=np.float64)
    _lib.check(L.cbgpu_histogram(_ptr(bins), n, F, B, _ptr(g), _ptr(h), _ptr(lo), n_leaves, _ptr(out)))
    return out


def select_borders(columns, border_count: int = 254, border_type: str = "GreedyLogSum",
                   nan_mode: str = "Min", device: int = 0):
    """Device border selection for every float column, as catboost-rs's builder
    derives them (builder.rs:1677-1720 -> cb_data::select_borders_f32).

    Returns one ascending f64 array per column, or None when the border type
    is one the device declines (the exact MinEntropy / MaxLogSum binarizers).
    """
    L = _lib.load()
    cols = [np.ascontiguousarray(c, dtype=np.float32) for c in columns]
    if not cols:
        raise ValueError("select_borders: no columns")
    n = cols[0].size
    if any(c.size != n for c in cols):
        raise ValueError("select_borders: columns differ in length")
    F = len(cols)
    ptrs = (C.c_void_p * F)(*[c.ctypes.data for c in cols])
    out = np.empty((F, max(int(border_count), 1)), dtype=np.float64)
    counts = np.zeros(F, dtype=np.int32)
    rc = L.cbgpu_select_borders(ptrs, n, F, int(border_count), BORDER_TYPE[border_type], NAN_MODE[nan_mode],
                                device, _ptr(out), _ptr(counts))
    if _lib.check(rc) == _lib.DECLINED:
        return None
    return [out[f, :counts[f]].copy() for f in range(F)]


def flatten_oblivious(split_feature, split_border, leaf_values):
    """CSR lowering of an oblivious ensemble, cb_model::flatten_oblivious_f64
    (crates/cb-model/src/gpu_apply.rs:120-193): split_feature [T, D] (-1 marks
    an unused level), split_border [T, D] border values, leaf_values [T, 2^D]
    learning-rate scaled (a tree with d splits owns its first 2^d values).
    Returns (split_features, split_borders, tree_split_offsets, leaf_values,
    tree_leaf_offsets)."""
    sf = np.asarray(split_feature)
    sb = np.asarray(split_border, dtype=np.float64)
    lv = np.asarray(leaf_values, dtype=np.float64)
    depth = (sf >= 0).sum(axis=1) if sf.size else np.zeros(sf.shape[0], dtype=np.int64)
    keep = sf >= 0
    so = np.concatenate([[0], np.cumsum(depth)]).astype(np.uint32)
    lo = np.concatenate([[0], np.cumsum(1 << depth.astype(np.int64))]).astype(np.uint32)
    leaves = np.concatenate([lv[t, : 1 << int(d)] for t, d in enumerate(depth)]) if sf.shape[0] else np.zeros(0)
    return (np.ascontiguousarray(sf[keep], dtype=np.uint32), np.ascontiguousarray(sb[keep], dtype=np.float64), so,
            np.ascontiguousarray(leaves, dtype=np.float64), lo)


def apply_oblivious(features_fm, flat, bias: float = 0.0, nan_above=None, device: int = 0) -> np.ndarray:
    """Raw predictions on the device (Model::predict_raw_on_device,
    crates/catboost-rs/src/model.rs:360-384): features_fm f32 [F][n]."""
    L = _lib.load()
    x = np.ascontiguousarray(features_fm, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("apply_oblivious: features must be [n_features][n]")
    F, n = x.shape
    # named, contiguous, correctly typed arrays stay alive across the call
    sf = np.ascontiguousarray(flat[0], dtype=np.uint32)
    sb = np.ascontiguousarray(flat[1], dtype=np.float64)
    so = np.ascontiguousarray(flat[2], dtype=np.uint32)
    lv = np.ascontiguousarray(flat[3], dtype=np.float64)
    lo = np.ascontiguousarray(flat[4], dtype=np.uint32)
    na = None if nan_above is None else np.ascontiguousarray(nan_above, dtype=np.uint8)
    if so.size < 1 or lo.size != so.size or sf.size != sb.size or (na is not None and na.size < F):
        raise ValueError("apply_oblivious: inconsistent flat model")
    out = np.empty(n, dtype=np.float64)
    _lib.check(L.cbgpu_apply_oblivious(_ptr(x), n, F, _ptr(sf), _ptr(sb), _ptr(so), so.size - 1, _ptr(lv), _ptr(lo),
                                       float(bias), _ptr(na), device, _ptr(out)))
    return out


def bootstrap_weights(kind: str, n: int, *, row_offset=0, rand_seed=0, rng_raw4=None, sample_rate=1.0,
                      bagging_temperature=1.0, der_obj=None, mvs_lambda=0.0) -> np.ndarray:
    """Device bootstrap weights (crates/cb-train/src/bootstrap.rs semantics)."""
    L = _lib.load()
    out = np.empty(n, dtype=np.float64)
    raw = None if rng_raw4 is None else np.ascontiguousarray(rng_raw4, dtype=np.uint64)
    d = None if der_obj is None else np.ascontiguousarray(der_obj, dtype=np.float64)
    _lib.check(L.cbgpu_bootstrap_weights(BOOT[kind], n, row_offset, rand_seed & (2**64 - 1), _ptr(raw),
                                         sample_rate, bagging_temperature, _ptr(d), mvs_lambda, _ptr(out)))
    return out
