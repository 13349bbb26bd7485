"""ctypes binding of libcbgpu.so (include/cbgpu.h).

The product path has exactly one implementation: the CUDA library.  Loading
fails loudly when the library is missing or no CUDA device is present; there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcbgpu.so")

OK, DECLINED, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_NCCL, ERR_DEVICE, ERR_NO_DEVICE = range(8)


class RankParams(C.Structure):
    _fields_ = [("l2_leaf_reg", C.c_double), ("softmax_lambda", C.c_double), ("softmax_beta", C.c_double),
                ("lambdamart_sigma", C.c_double), ("lambdamart_top", C.c_int64), ("lambdamart_norm", C.c_int32),
                ("lambdamart_metric", C.c_int32), ("yeti_permutations", C.c_int32), ("yeti_decay", C.c_double),
                ("srank_metric", C.c_int32), ("srank_num_estimations", C.c_int32), ("srank_sigma", C.c_double),
                ("srank_mu", C.c_double), ("pair_weight", C.c_void_p)]


class BeginArgs(C.Structure):
    _fields_ = [
        ("loss", C.c_int32), ("depth", C.c_int32), ("boosting_type_is_plain", C.c_int32),
        ("fold_count", C.c_int32), ("score_function", C.c_int32), ("n", C.c_int64),
        ("n_features", C.c_int32), ("n_bins", C.c_int32), ("learning_rate", C.c_double),
        ("scaled_l2", C.c_double), ("weight", C.c_void_p), ("grow_policy", C.c_int32),
        ("bootstrap_type", C.c_int32), ("sample_rate", C.c_float), ("bagging_temperature", C.c_float),
        ("has_mvs_lambda", C.c_int32), ("mvs_lambda", C.c_double), ("rng_seed", C.c_uint64),
        ("bias", C.c_double), ("sample_from_host", C.c_int32), ("random_strength", C.c_double),
        ("device", C.c_int32), ("rank", C.c_int32), ("world_size", C.c_int32),
        ("row_offset", C.c_int64), ("n_total", C.c_int64), ("nccl_unique_id", C.c_void_p),
        ("border_counts", C.c_void_p), ("exact_leaf", C.c_int32), ("quantile_alpha", C.c_double),
        ("quantile_delta", C.c_double),
    ]


EXPORTS = [
    "cbgpu_begin", "cbgpu_begin_raw", "cbgpu_grow_tree", "cbgpu_end", "cbgpu_stage_sample",
    "cbgpu_compute_gradients",
    "cbgpu_last_error", "cbgpu_session_approx", "cbgpu_session_bins", "cbgpu_session_last_sample",
    "cbgpu_session_timing", "cbgpu_session_timing_sum", "cbgpu_session_set_profiling", "cbgpu_session_set_graphs", "cbgpu_session_rng_state",
    "cbgpu_histogram", "cbgpu_bootstrap_weights", "cbgpu_nccl_unique_id", "cbgpu_version",
    "cbgpu_session_mark", "cbgpu_session_elapsed_ms", "cbgpu_histogram_noalloc",
    "cbgpu_rank_feature_slice", "cbgpu_rank_select_split", "cbgpu_rank_mvs_partial",
    "cbgpu_select_borders", "cbgpu_apply_oblivious",
    "cbgpu_multi_begin_raw", "cbgpu_multi_begin_cat_raw", "cbgpu_multi_grow_tree", "cbgpu_multi_approx", "cbgpu_multi_end",
    "cbgpu_rank_begin_raw",
]

_lib = None


class CbGpuError(RuntimeError):
    """A non-OK, non-declined status from the C ABI (the CbError analogue)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"cbgpu status {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH):
    """Load libcbgpu.so and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m catboost_rs_b200.build`")
    L = C.CDLL(path)
    vp, i32, i64, u64, f64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_double, C.c_float
    sig = {
        "cbgpu_begin": ([C.POINTER(BeginArgs), vp, C.POINTER(vp)], C.c_int),
        "cbgpu_begin_raw": ([C.POINTER(BeginArgs), vp, vp, vp, C.POINTER(vp)], C.c_int),
        "cbgpu_grow_tree": ([vp, vp, vp, i64, vp, i64, vp, vp, vp, vp, vp, i32], C.c_int),
        "cbgpu_end": ([vp], C.c_int),
        "cbgpu_stage_sample": ([vp, vp, i64], C.c_int),
        "cbgpu_compute_gradients": ([i32, vp, vp, i64, vp, vp], C.c_int),
        "cbgpu_last_error": ([], C.c_char_p),
        "cbgpu_session_approx": ([vp, vp, i64], C.c_int),
        "cbgpu_session_bins": ([vp, vp, i64, i32], C.c_int),
        "cbgpu_session_last_sample": ([vp, vp, i64], C.c_int),
        "cbgpu_session_timing": ([vp, vp], C.c_int),
        "cbgpu_session_timing_sum": ([vp, vp, i32], C.c_int),
        "cbgpu_session_set_profiling": ([vp, i32], C.c_int),
        "cbgpu_session_set_graphs": ([vp, i32], C.c_int),
        "cbgpu_session_rng_state": ([vp, vp], C.c_int),
        "cbgpu_session_mark": ([vp, i32], C.c_int),
        "cbgpu_session_elapsed_ms": ([vp, i32, i32, vp], C.c_int),
        "cbgpu_histogram": ([vp, i64, i32, i32, vp, vp, vp, i32, vp], C.c_int),
        "cbgpu_bootstrap_weights": ([i32, i64, i64, u64, vp, f32, f32, vp, f64, vp], C.c_int),
        "cbgpu_histogram_noalloc": ([vp, i64, i32, i32, i32, vp, vp, vp, vp], C.c_int),
        "cbgpu_rank_feature_slice": ([i32, i32, i32, vp, vp], C.c_int),
        "cbgpu_rank_select_split": ([i32, i32, i32, vp, vp, vp, vp, vp, vp], C.c_int),
        "cbgpu_rank_mvs_partial": ([i32, i64, vp, f64, vp, vp, f64, vp], C.c_int),
        "cbgpu_select_borders": ([vp, i64, i32, i32, i32, i32, i32, vp, vp], C.c_int),
        "cbgpu_apply_oblivious": ([vp, i64, i32, vp, vp, vp, i32, vp, vp, f64, vp, i32, vp], C.c_int),
        "cbgpu_multi_begin_raw": ([C.POINTER(BeginArgs), i32, vp, vp, vp, C.POINTER(vp)], C.c_int),
        "cbgpu_multi_begin_cat_raw": ([C.POINTER(BeginArgs), i32, vp, vp, vp, i32, vp, C.POINTER(vp)], C.c_int),
        "cbgpu_multi_grow_tree": ([vp, vp, vp, i64, vp, i64, vp, vp, vp, vp, vp, i32], C.c_int),
        "cbgpu_multi_approx": ([vp, vp, i64], C.c_int),
        "cbgpu_rank_begin_raw": ([C.POINTER(BeginArgs), vp, i32, vp, vp, i64, C.POINTER(RankParams), vp, vp, vp,
                                  C.POINTER(vp)], C.c_int),
        "cbgpu_multi_end": ([vp], C.c_int),
        "cbgpu_nccl_unique_id": ([vp], C.c_int),
        "cbgpu_version": ([], C.c_char_p),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def last_error() -> str:
    return load().cbgpu_last_error().decode()


def check(rc: int) -> int:
    if rc not in (OK, DECLINED):
        raise CbGpuError(rc, last_error())
    return rc
