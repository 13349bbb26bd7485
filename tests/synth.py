"""Seeded synthetic inputs shaped like the BASELINE configs, at test sizes.

Borders are uniform quantiles of each column (numpy), with the nan_mode=Min
sentinel f32::MIN prepended to NaN-bearing columns (cb-data nan_mode.rs
insert_sentinel); both the device and the oracle consume the same borders.
"""
from __future__ import annotations

import numpy as np

FMIN = float(np.finfo(np.float32).min)


def quantile_borders(col: np.ndarray, border_count: int) -> np.ndarray:
    v = col[~np.isnan(col)].astype(np.float64)
    has_nan = np.isnan(col).any()
    k = border_count - 1 if has_nan else border_count
    if v.size == 0 or k <= 0:
        b = np.zeros(0)
    else:
        qs = np.quantile(v, np.linspace(0, 1, k + 2)[1:-1])
        b = np.unique(qs.astype(np.float32).astype(np.float64))
    if has_nan:
        b = np.concatenate([[FMIN], b])
    return b


def make_dataset(n, F, *, seed=0, nan_frac=0.0, loss="RMSE", border_count=32, uniform_half=False):
    rs = np.random.RandomState(seed)
    X = rs.standard_normal((n, F)).astype(np.float32)
    if uniform_half:
        X[:, F // 2:] = rs.uniform(0, 1, (n, F - F // 2)).astype(np.float32)
    if nan_frac > 0:
        m = rs.uniform(size=(n, F)) < nan_frac
        X[m] = np.nan
    w = np.zeros(F)
    idx = rs.choice(F, size=min(F, 10), replace=False)
    w[idx] = rs.standard_normal(idx.size)
    Xz = np.nan_to_num(X.astype(np.float64))
    z = Xz @ w
    if loss == "RMSE":
        y = z + 0.1 * rs.standard_normal(n)
    else:
        zz = z + 0.5 * Xz[:, idx[0]] * Xz[:, idx[1 % idx.size]]
        y = (rs.uniform(size=n) < 1.0 / (1.0 + np.exp(-zz))).astype(np.float64)
    borders = [quantile_borders(X[:, f], border_count) for f in range(F)]
    return X, y, borders
