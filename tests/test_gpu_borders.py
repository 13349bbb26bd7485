"""Device border selection (cbgpu_select_borders) against upstream and the oracle.

The device restates the reference's binarizers (crates/cb-data/src/borders.rs,
border_types.rs) and the builder's per-column NaN rule
(crates/catboost-rs/src/builder.rs:1677-1720).  Borders are f32 values, so the
bar is exact equality: with the upstream CatBoost 1.2.10 border sets the
reference's own border tests use (tests/golden/borders.npz), and with the CPU
oracle on synthetic columns that exercise the 200,000-row sample, NaNs under
both sentinel modes, heavy duplicate runs, signed zeros and degenerate columns.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "borders.npz")
DEVICE_TYPES = ("GreedyLogSum", "GreedyMinEntropy", "Median", "Uniform", "UniformAndQuantiles")


@pytest.fixture(scope="module")
def cb():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    cb.load_library()
    return cb


def _f32_equal(a, b):
    return a.size == b.size and np.array_equal(np.asarray(a).astype(np.float32), np.asarray(b).astype(np.float32))


def test_device_borders_match_upstream_sets(cb):
    z = np.load(GOLDEN)
    cells = [c for c in json.loads(str(z["cells"])) if c["border_type"] in DEVICE_TYPES]
    assert len(cells) >= 40
    for c in cells:
        X = z[f"X__{c['dataset']}"]
        flat, counts = z[f"B__{c['stem']}"], z[f"C__{c['stem']}"]
        offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        got = cb.select_borders([X[:, f] for f in range(X.shape[1])], c["border_count"], c["border_type"],
                                c["nan_mode"])
        for f in range(X.shape[1]):
            want = flat[offs[f]:offs[f + 1]]
            assert _f32_equal(got[f], want), (c["stem"], f, got[f][:6], want[:6])
            # the device returns exactly the oracle's f64 values
            o = oracle.select_borders(X[:, f], c["border_count"], c["border_type"], c["nan_mode"])
            assert np.array_equal(got[f], o), (c["stem"], f)


def _synthetic(n, seed):
    rs = np.random.RandomState(seed)
    cols = [
        rs.standard_normal(n).astype(np.float32),                       # N(0,1) with NaNs below
        rs.uniform(size=n).astype(np.float32),                          # U(0,1)
        np.round(rs.standard_normal(n), 1).astype(np.float32),          # heavy duplicate runs
        np.full(n, 3.25, np.float32),                                   # constant
        np.where(rs.uniform(size=n) < 0.5, -0.0, 0.0).astype(np.float32) + (rs.uniform(size=n) < 0.1),
        rs.zipf(1.5, n).clip(max=500).astype(np.float32),               # few, skewed values
        (rs.lognormal(size=n) * 1e6).astype(np.float32),                # wide dynamic range
    ]
    cols[0][rs.uniform(size=n) < 0.05] = np.nan
    cols[5][: n // 100] = np.nan
    return cols


@pytest.mark.parametrize("n", [0, 1, 2, 1000, 199_999, 300_001])
def test_device_borders_match_oracle_synthetic(cb, n):
    cols = _synthetic(n, 7 + n % 13)
    grid = [(t, 128, m) for t in DEVICE_TYPES for m in ("Min", "Max")]
    grid += [("GreedyLogSum", 16, "Min"), ("GreedyLogSum", 254, "Min"), ("Median", 254, "Max"),
             ("GreedyLogSum", 1, "Min"), ("Uniform", 2, "Max")]
    for t, bc, mode in grid:
        got = cb.select_borders(cols, bc, t, mode)
        assert len(got) == len(cols)
        for f, col in enumerate(cols):
            want = oracle.select_borders(col, bc, t, mode)
            assert np.array_equal(got[f], want), (n, t, bc, mode, f, got[f][:5], want[:5])
            assert got[f].size <= bc


def test_all_nan_column_and_sentinels(cb):
    n = 5000
    col = np.full(n, np.nan, np.float32)
    mixed = np.random.RandomState(1).standard_normal(n).astype(np.float32)
    mixed[::9] = np.nan
    fmax = float(np.finfo(np.float32).max)
    lo = cb.select_borders([col, mixed], 32, "GreedyLogSum", "Min")
    hi = cb.select_borders([col, mixed], 32, "GreedyLogSum", "Max")
    assert np.array_equal(lo[0], [-fmax]) and np.array_equal(hi[0], [fmax])
    assert lo[1][0] == -fmax and hi[1][-1] == fmax and lo[1].size == 32 and hi[1].size == 32
    assert np.array_equal(lo[1][1:], hi[1][:-1])


def test_errors_and_declines(cb):
    from catboost_rs_b200 import CbGpuError
    col = np.array([1.0, np.nan, 2.0], np.float32)
    with pytest.raises(CbGpuError, match="nan_mode"):
        cb.select_borders([col], 8, "GreedyLogSum", "Forbidden")
    assert cb.select_borders([col], 8, "MaxLogSum", "Min") is None
    assert cb.select_borders([col], 8, "MinEntropy", "Min") is None
    with pytest.raises(CbGpuError):
        cb.select_borders([col], 0, "GreedyLogSum", "Min")
    with pytest.raises(CbGpuError):
        cb.select_borders([col], 1025, "GreedyLogSum", "Min")
    # NaN-free under Forbidden is fine
    assert cb.select_borders([np.array([1.0, 2.0, 3.0], np.float32)], 8, "GreedyLogSum", "Forbidden")[0].size == 2


def test_config2_shape_sample(cb):
    # config 2's feature mix at a row count over the 200k cap: every border set
    # (128 borders, nan_mode=Min sentinel on NaN columns) equals the oracle's
    rs = np.random.RandomState(11)
    n, F = 600_000, 8
    cols = [rs.standard_normal(n).astype(np.float32) if f % 2 == 0 else rs.uniform(size=n).astype(np.float32)
            for f in range(F)]
    for c in cols:
        c[rs.uniform(size=n) < 0.05] = np.nan
    got = cb.select_borders(cols, 128, "GreedyLogSum", "Min")
    for f in range(F):
        want = oracle.select_borders(cols[f], 128, "GreedyLogSum", "Min")
        assert want.size == 128 and np.array_equal(got[f], want), f
