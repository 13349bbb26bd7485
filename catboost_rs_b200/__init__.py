"""catboost_rs_b200 -- B200-native oblivious-tree training path for catboost_rs.

The compute is libcbgpu.so (CUDA for sm_100a behind the C ABI in
include/cbgpu.h).  This package holds the host-side mirror of the reference's
`cb_compute::Runtime` seam (runtime.py), the boosting loop that drives it
(boosting.py) and the build script (build.py).
"""
from ._lib import CbGpuError, load as load_library  # noqa: F401
from .runtime import (B200MultiRuntime, B200Runtime, DeviceGrownTree, DeviceTrainConfig, Derivatives,  # noqa: F401
                      apply_oblivious, bootstrap_weights, flatten_oblivious, histogram, nccl_unique_id,
                      select_borders)
from .boosting import (FitParams, MultiClassModel, ObliviousModel, RankingModel, fit,  # noqa: F401
                       fit_multiclass, fit_ranking, normalize_leaf_values, perfect_hash_bins, seq_sum, starting_approx)

__version__ = "0.1.0"
from . import model_json  # noqa: F401,E402
from .model_json import from_json, load_json, save_json, to_json  # noqa: F401,E402
from . import model_cbm  # noqa: F401,E402
from .model_cbm import load_cbm, save_cbm  # noqa: F401,E402
