"""Device ensemble apply (cbgpu_apply_oblivious) against the oracle and upstream.

The device apply restates the reference's CPU apply (crates/cb-model/src/
apply.rs:150-173, 374-410) over the CSR lowering of flatten_oblivious_f64
(crates/cb-model/src/gpu_apply.rs:120-193); it must equal the oracle's apply
bit for bit (same comparisons, same tree-order sum), and through it upstream
CatBoost 1.2.10's predictions at the reference's 1e-5 bar.
"""
import json
import os

import numpy as np
import pytest

from golden_io import load_scenario, scenario_names
from oracle import oracle

pytestmark = pytest.mark.gpu

PRED_TOL = 1e-5
FMAX = float(np.finfo(np.float32).max)


@pytest.fixture(scope="module")
def cb():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    cb.load_library()
    return cb


def _random_ensemble(rs, T, depth, F, extra_features=0, short_leaves=False):
    sf = rs.randint(0, F + extra_features, size=(T, depth)).astype(np.int32)
    sb = rs.standard_normal((T, depth))
    lv = rs.standard_normal((T, 1 << depth)) * 0.1
    # ragged trees: some stop early (-1 marks an unused level)
    for t in range(0, T, 7):
        d = rs.randint(0, depth + 1)
        sf[t, d:] = -1
    flat = list(oracle.flatten_oblivious(sf, sb, lv))
    if short_leaves:  # a leaf array shorter than its splits address: those leaves add 0
        so, leaves, lo = flat[2], flat[3], flat[4]
        keep = np.ones(leaves.size, bool)
        for t in range(0, so.size - 1, 5):
            keep[lo[t + 1] - 1] = False
        new_lo = np.concatenate([[0], np.cumsum([keep[lo[t]:lo[t + 1]].sum() for t in range(so.size - 1)])])
        flat[3], flat[4] = leaves[keep], new_lo.astype(np.uint32)
    return tuple(flat)


def test_fixture_models_match_oracle_and_upstream(cb):
    for name in scenario_names():
        sc = load_scenario(name)
        flat = cb.flatten_oblivious(sc["split_feature"], sc["split_border"], sc["leaf_values"])
        oflat = oracle.flatten_oblivious(sc["split_feature"], sc["split_border"], sc["leaf_values"])
        for a, b in zip(flat, oflat):
            np.testing.assert_array_equal(a, b)
        na = np.array([len(b) > 0 and b[-1] == FMAX for b in sc["borders"]], dtype=np.uint8)
        X = sc["X"].T.copy()
        bias = 0.25
        got = cb.apply_oblivious(X, flat, bias, na)
        want = oracle.apply_oblivious(X, oflat, bias, na)
        np.testing.assert_array_equal(got, want)
        if "preds_eval" in sc:
            Xe = sc["X_eval"].T.copy()
            np.testing.assert_array_equal(cb.apply_oblivious(Xe, flat, bias, na),
                                          oracle.apply_oblivious(Xe, oflat, bias, na))


@pytest.mark.parametrize("n,F,T,depth", [(1, 1, 1, 1), (100_001, 37, 300, 8), (5000, 250, 100, 6),
                                         (3000, 2100, 40, 10), (70_000, 3, 30, 16)])
def test_random_ensembles_match_oracle(cb, n, F, T, depth):
    rs = np.random.RandomState(n + F)
    X = rs.standard_normal((F, n)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.05] = np.nan
    X[rs.uniform(size=X.shape) < 0.01] = -0.0
    flat = _random_ensemble(rs, T, depth, F, extra_features=2, short_leaves=True)
    na = (rs.uniform(size=F) < 0.5).astype(np.uint8)
    for nan_above in (None, na):
        got = cb.apply_oblivious(X, flat, -1.5, nan_above)
        want = oracle.apply_oblivious(X, flat, -1.5, nan_above)
        np.testing.assert_array_equal(got, want)


def test_edge_models(cb):
    X = np.array([[np.nan, -1.0, 0.5, 2.0]], dtype=np.float32)
    empty = (np.zeros(0, np.uint32), np.zeros(0), np.array([0], np.uint32), np.zeros(0), np.array([0], np.uint32))
    z = cb.apply_oblivious(X, empty, -0.0)
    assert np.array_equal(z, np.zeros(4)) and not np.any(np.signbit(z))
    const = (np.zeros(0, np.uint32), np.zeros(0), np.array([0, 0], np.uint32), np.array([2.5]),
             np.array([0, 1], np.uint32))
    assert cb.apply_oblivious(X, const, 1.0).tolist() == [3.5] * 4
    one = (np.array([0], np.uint32), np.array([0.0]), np.array([0, 1], np.uint32), np.array([10.0, 20.0]),
           np.array([0, 2], np.uint32))
    assert cb.apply_oblivious(X, one, 1.0).tolist() == [11.0, 11.0, 21.0, 21.0]
    assert cb.apply_oblivious(X, one, 1.0, np.array([1], np.uint8)).tolist() == [21.0, 11.0, 21.0, 21.0]
    assert cb.apply_oblivious(np.zeros((1, 0), np.float32), one, 1.0).size == 0
    from catboost_rs_b200 import CbGpuError
    deep = (np.zeros(17, np.uint32), np.zeros(17), np.array([0, 17], np.uint32), np.zeros(1 << 17),
            np.array([0, 1 << 17], np.uint32))
    with pytest.raises(CbGpuError):
        cb.apply_oblivious(X, deep, 0.0)
    bad = (np.array([0], np.uint32), np.array([0.0]), np.array([1, 1], np.uint32), np.array([1.0, 2.0]),
           np.array([0, 2], np.uint32))
    with pytest.raises(CbGpuError):
        cb.apply_oblivious(X, bad, 0.0)


def test_two_chunks(cb):
    # more than 1 GiB of features: the rows go through two staged chunks
    rs = np.random.RandomState(3)
    n, F = 2_800_000, 100
    X = np.random.default_rng(3).standard_normal((F, n), dtype=np.float32)
    flat = _random_ensemble(rs, 20, 6, F)
    got = cb.apply_oblivious(X, flat, 0.5)
    want = oracle.apply_oblivious(X, flat, 0.5)
    np.testing.assert_array_equal(got, want)


def test_fit_then_predict(cb):
    # a device fit's predictions on its training rows equal its resident approximant
    rs = np.random.RandomState(5)
    n, F = 20000, 10
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.03] = np.nan
    y = np.nan_to_num(X[:, 0]) - 2 * np.nan_to_num(X[:, 1]) + 0.1 * rs.standard_normal(n)  # a finite target
    borders = [np.concatenate([[-FMAX], np.unique(np.quantile(X[~np.isnan(X[:, f]), f],
                                                              np.linspace(0, 1, 34)[1:-1]).astype(np.float32))
                               .astype(np.float64)]) for f in range(F)]
    fp = cb.FitParams(loss="RMSE", depth=6, iterations=20, learning_rate=0.1)
    m = cb.fit([X[:, f].copy() for f in range(F)], borders, y, fp, staged=True)
    pred = m.predict(X)
    assert np.max(np.abs(pred - m.staged[-1])) <= 1e-9
    o = oracle.apply_oblivious(X.T.copy(), oracle.flatten_oblivious(m.split_feature, m.split_borders(),
                                                                      m.leaf_values), m.bias)
    np.testing.assert_array_equal(pred, o)


@pytest.mark.parametrize("name", ["regression_skeleton", "binclf_skeleton", "nan_mode_Max", "nan_mode_Min"])
def test_model_json_predict_on_device(cb, name):
    # an upstream model.json read by the package's reader and applied on the device
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "model_json.npz"))
    m = cb.from_json(json.loads(str(z[name])))
    sc = load_scenario(name)
    X, want = (sc["X_eval"], sc["preds_eval"]) if name.startswith("nan_mode") else (sc["X"], sc["staged"][-1])
    got = m.predict(X)
    assert np.max(np.abs(got - want)) <= 1e-5
