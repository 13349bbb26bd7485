"""Exact leaves (MAE / Quantile) on the scalar device session against the oracle.

The structure comes from quantile_der1 (crates/cb-compute/src/loss.rs:166-193)
through the same histogram / score kernels as RMSE; the leaf values are each
leaf's weighted alpha-quantile of the f32 residuals with the delta adjustment
(crates/cb-compute/src/leaf.rs:445-520), computed on the device by a
(leaf, residual) radix sort and one block per leaf.  The upstream fixtures run
through test_gpu_parity.py's fixture test.  The synthetic cases use dyadic
alphas and integer weights: every der and weight sum is then exact in f64 on
both sides, so exactly tied split scores resolve the same way.
"""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def cb():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import catboost_rs_b200 as cb
    cb.load_library()
    return cb


CASES = [
    dict(loss="MAE", alpha=0.5, n=30000, F=10, depth=6, score="Cosine", w=False, it=5),
    dict(loss="Quantile", alpha=0.25, n=20000, F=8, depth=5, score="L2", w=True, it=5),
    dict(loss="Quantile", alpha=0.875, n=70001, F=6, depth=4, score="Cosine", w=False, it=4),
    dict(loss="Quantile", alpha=0.0, n=5000, F=5, depth=3, score="L2", w=False, it=3),
    dict(loss="Quantile", alpha=0.5, n=3000, F=4, depth=10, score="Cosine", w=True, it=3),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['loss']}-a{c['alpha']}-d{c['depth']}-n{c['n']}")
def test_exact_leaf_matches_oracle(cb, case):
    rs = np.random.RandomState(case["n"] + case["depth"])
    n, F = case["n"], case["F"]
    X = rs.standard_normal((n, F)).astype(np.float32)
    X[rs.uniform(size=X.shape) < 0.02] = np.nan
    y = np.nan_to_num(X[:, 0]) * 2 + np.sin(np.nan_to_num(X[:, 1])) + rs.standard_t(3, n)
    w = rs.randint(1, 4, n).astype(np.float64) if case["w"] else None
    borders = [oracle.select_borders(X[:, f], 32) for f in range(F)]
    fp = cb.FitParams(loss=case["loss"], depth=case["depth"], iterations=case["it"], learning_rate=0.3,
                      score_function=case["score"], boost_from_average=False, leaf_estimation_method="Exact",
                      quantile_alpha=case["alpha"], quantile_delta=1e-6)
    m = cb.fit([X[:, f].copy() for f in range(F)], borders, y, fp, weights=w, staged=True)
    bins = oracle.quantize(X.T.copy(), borders)
    o = oracle.train(bins, [len(b) for b in borders], y, loss=case["loss"], depth=fp.depth,
                     iterations=fp.iterations, learning_rate=fp.learning_rate, l2_leaf_reg=fp.l2_leaf_reg,
                     score_function=fp.score_function, boost_from_average=False, weights=w,
                     leaf_estimation_method="Exact", quantile_alpha=case["alpha"], quantile_delta=1e-6)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= TOL
    assert np.max(np.abs(m.staged - o.staged)) <= TOL


def test_exact_leaf_declines(cb):
    rs = np.random.RandomState(2)
    n, F = 2000, 3
    X = rs.standard_normal((n, F)).astype(np.float32)
    borders = [oracle.select_borders(X[:, f], 16) for f in range(F)]
    cols = [X[:, f].copy() for f in range(F)]
    nb = max(len(b) for b in borders) + 1

    def begin(loss, exact, **kw):
        rt = cb.B200Runtime()
        cfg = cb.DeviceTrainConfig(exact_leaf=exact, **kw)
        return rt, rt.begin_device_training_raw(loss, 3, True, 1, "L2", cols, borders, None, n, F, nb, 0.1, 3.0, cfg)

    for loss, exact, kw in (("MAE", False, {}), ("Quantile", False, {}), ("RMSE", True, {}),
                            ("Logloss", True, {}), ("MAE", True, dict(bootstrap_type="Bernoulli", sample_rate=0.5))):
        rt, ok = begin(loss, exact, **kw)
        assert not ok and rt.decline_reason, (loss, exact, kw)
    rt, ok = begin("Quantile", True, quantile_alpha=0.5)
    assert ok
    rt.end_device_training()
