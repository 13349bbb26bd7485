"""Parity of the CUDA path (through the C ABI) against the CPU oracle and the
upstream fixtures.  Bars: bins, leaf ids and bootstrap
weights bit-exact; histogram sums within 1e-6 relative; identical trees except
at near-ties; predictions within 1e-5.
"""
import numpy as np
import pytest

import oracle
from golden_io import load_scenario, scenario_names
from synth import make_dataset

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("catboost_rs_b200")

HIST_RTOL = 1e-6   # histogram sums, relative to the sum of |contributions|
PRED_TOL = 1e-5    # leaf values / staged approximants / predictions


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _cols(X):
    return [np.ascontiguousarray(X[:, f]) for f in range(X.shape[1])]


# ---- quantization: bit-exact ----------------------------------------------

@pytest.mark.parametrize("nan_mode", ["Min", "Max"])
def test_device_quantization_bit_exact(nan_mode):
    X, y, borders = make_dataset(5003, 37, seed=3, nan_frac=0.05, border_count=64)
    if nan_mode == "Max":
        fmax = float(np.finfo(np.float32).max)
        borders = [np.concatenate([b[1:], [fmax]]) if b.size and b[0] < -1e38 else b for b in borders]
    rt = cb.B200Runtime()
    cfg = cb.DeviceTrainConfig()
    assert rt.begin_device_training_raw("RMSE", 4, True, 1, "L2", _cols(X), borders, None, X.shape[0],
                                        X.shape[1], max(len(b) for b in borders) + 1, 0.1, 3.0, cfg)
    dev = rt.device_bins(X.shape[1])
    rt.end_device_training()
    ref = oracle.quantize(X.T.copy(), borders)
    np.testing.assert_array_equal(dev, ref)


# ---- histogram: 1e-6 relative ---------------------------------------------

@pytest.mark.parametrize("n,F,B,leaves", [(0, 5, 8, 1), (1, 3, 4, 1), (33, 33, 17, 2), (20000, 50, 129, 8),
                                          (70001, 64, 256, 4)])
def test_histogram_matches_oracle(n, F, B, leaves):
    rs = np.random.RandomState(n + F)
    bins = rs.randint(0, B, size=(n, F)).astype(np.uint8)
    if n > 10:
        bins[: n // 10, 0] = 0  # a hot bin (the NaN bin analogue)
    g = rs.standard_normal(n) * rs.exponential(1.0, n)
    h = rs.exponential(1.0, n)
    leaf = rs.randint(0, leaves, size=n).astype(np.int32)
    dev = cb.histogram(bins, g, h, leaf, leaves, B)
    ref = oracle.build_histogram(bins.T.copy(), g, h, leaf, leaves, B)
    mag = oracle.build_histogram(bins.T.copy(), np.abs(g), np.abs(h), leaf, leaves, B)
    assert dev.shape == ref.shape
    assert np.all(np.abs(dev - ref) <= HIST_RTOL * mag + 1e-300)
    # exact integer accumulation: the result does not depend on the order
    dev2 = cb.histogram(bins, g, h, leaf, leaves, B)
    np.testing.assert_array_equal(dev, dev2)


# ---- bootstrap weights: bit-exact -------------------------------------------

@pytest.mark.parametrize("temp", [1.0, 0.5])
@pytest.mark.parametrize("n,offset", [(1, 0), (999, 0), (1000, 0), (25037, 0), (4000, 3000)])
def test_bayesian_weights_bit_exact(temp, n, offset):
    r = oracle.TFastRng64(7)
    total = offset + n
    sw, _ = oracle.bootstrap("Bayesian", np.zeros(total), r, bagging_temperature=temp)
    r2 = oracle.TFastRng64(7)
    seed = r2.gen_rand()
    dev = cb.bootstrap_weights("Bayesian", n, row_offset=offset, rand_seed=seed, bagging_temperature=temp)
    if temp == 1.0:
        # the bench configuration: pow(w, 1) == w, every weight bit-exact
        np.testing.assert_array_equal(dev, sw[offset:])
    else:
        # T != 1: the device pow (rounded to f32) may differ from glibc powf by
        # one f32 ulp; the RNG stream and FastLogf part stay bit-exact.
        ulp = np.spacing(np.abs(sw[offset:]).astype(np.float32)).astype(np.float64)
        assert np.all(np.abs(dev - sw[offset:]) <= ulp)


@pytest.mark.parametrize("n,offset", [(1, 0), (12345, 0), (5000, 777)])
def test_bernoulli_mask_bit_exact(n, offset):
    r = oracle.TFastRng64(11)
    r.gen_rand()
    base = r.raw_state()
    total = offset + n
    _, ctl = oracle.bootstrap("Bernoulli", np.zeros(total), r, subsample=0.66)
    dev = cb.bootstrap_weights("Bernoulli", n, row_offset=offset, rng_raw4=base, sample_rate=0.66)
    np.testing.assert_array_equal(dev, ctl[offset:].astype(np.float64))


@pytest.mark.parametrize("n", [1, 100, 8192, 8193, 30000])
def test_mvs_weights_bit_exact(n):
    rs = np.random.RandomState(n)
    der = np.abs(rs.standard_normal(n) * rs.exponential(1.0, n))
    r = oracle.TFastRng64(5)
    prev = 0.37
    sw, _ = oracle.bootstrap("MVS", der, r, subsample=0.8, prev_leaf_mean=prev)
    r2 = oracle.TFastRng64(5)
    seed = r2.gen_rand()
    dev = cb.bootstrap_weights("MVS", n, rand_seed=seed, sample_rate=0.8, der_obj=der, mvs_lambda=prev * prev)
    np.testing.assert_array_equal(dev, sw)


# ---- gradients ------------------------------------------------------------

@pytest.mark.parametrize("loss", ["RMSE", "Logloss"])
def test_compute_gradients(loss):
    rs = np.random.RandomState(1)
    a = rs.standard_normal(1001) * 3
    t = (rs.uniform(size=1001) < 0.5).astype(np.float64) if loss == "Logloss" else rs.standard_normal(1001)
    d = cb.B200Runtime().compute_gradients(loss, a, t)
    r1, r2 = oracle.compute_gradients(loss, a, t)
    np.testing.assert_allclose(d.der1, r1, rtol=0, atol=1e-15)
    np.testing.assert_allclose(d.der2, r2, rtol=0, atol=1e-15)


# ---- whole fits against the upstream fixtures ------------------------------

DEVICE_SCENARIOS = [s for s in scenario_names() if "random_strength" not in s]


@pytest.mark.parametrize("name", DEVICE_SCENARIOS)
def test_device_fit_matches_upstream_fixture(name):
    sc = load_scenario(name)
    p = sc["params"]
    fp = cb.FitParams(loss=p["loss"], depth=p["depth"], iterations=p["iterations"],
                      learning_rate=p["learning_rate"], l2_leaf_reg=p["l2_leaf_reg"],
                      score_function=p["score_function"], bootstrap_type=p["bootstrap_type"],
                      subsample=p["subsample"], bagging_temperature=p["bagging_temperature"],
                      random_seed=p["random_seed"], boost_from_average=p["boost_from_average"],
                      leaf_estimation_method=p.get("leaf_estimation_method", "Gradient"),
                      quantile_alpha=p.get("quantile_alpha", 0.5), quantile_delta=p.get("quantile_delta", 1e-6))
    X = sc["X"]
    m = cb.fit(_cols(X), sc["borders"], sc["y"], fp, weights=sc.get("weights"), staged=True)
    np.testing.assert_array_equal(m.split_feature, sc["split_feature"])
    assert np.max(np.abs(m.split_borders() - sc["split_border"])) <= PRED_TOL
    assert np.max(np.abs(m.leaf_values - sc["leaf_values"])) <= PRED_TOL
    if "staged" in sc:
        assert np.max(np.abs(m.staged - sc["staged"])) <= PRED_TOL
    if "predictions" in sc:
        assert np.max(np.abs(m.staged[-1] - sc["predictions"])) <= PRED_TOL
    if "preds_eval" in sc:
        assert np.max(np.abs(m.predict(sc["X_eval"]) - sc["preds_eval"])) <= PRED_TOL


# ---- whole fits against the oracle on synthetic data ------------------------

def _oracle_fit(X, y, borders, fp, weights=None):
    bins = oracle.quantize(X.T.copy(), borders)
    return oracle.train(bins, [len(b) for b in borders], y, loss=fp.loss, depth=fp.depth,
                        iterations=fp.iterations, learning_rate=fp.learning_rate,
                        l2_leaf_reg=fp.l2_leaf_reg, score_function=fp.score_function,
                        bootstrap_type=fp.bootstrap_type, subsample=fp.subsample,
                        bagging_temperature=fp.bagging_temperature, random_seed=fp.random_seed,
                        boost_from_average=fp.boost_from_average, weights=weights, staged=True)


CASES = [
    dict(n=3000, F=12, loss="RMSE", depth=4, boot="No", score="L2", nan=0.0, it=6),
    dict(n=20000, F=40, loss="Logloss", depth=6, boot="Bayesian", score="Cosine", nan=0.05, it=8),
    dict(n=20000, F=30, loss="RMSE", depth=5, boot="Bernoulli", score="Cosine", nan=0.0, it=8),
    dict(n=40000, F=20, loss="RMSE", depth=6, boot="MVS", score="L2", nan=0.02, it=6),
    dict(n=9000, F=50, loss="Logloss", depth=8, boot="Bayesian", score="Cosine", nan=0.05, it=4),
    dict(n=2048, F=5, loss="CrossEntropy", depth=10, boot="No", score="Cosine", nan=0.0, it=3),
    # past 256 parents the partition reserves one slot per row, past 1024
    # leaves the final route adds leaf sums with global atomics
    dict(n=30000, F=8, loss="RMSE", depth=12, boot="Bayesian", score="Cosine", nan=0.02, it=2),
    # few rows per (chunk, tile) item at every level (as on one shard of a
    # multi-GPU fit): 4096-row chunks, and 64- + 32- + 4-feature tiles
    dict(n=200000, F=100, loss="Logloss", depth=8, boot="Bayesian", score="Cosine", nan=0.05, it=2),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['loss']}-{c['boot']}-d{c['depth']}-n{c['n']}")
def test_device_fit_matches_oracle(case):
    X, y, borders = make_dataset(case["n"], case["F"], seed=case["n"], nan_frac=case["nan"],
                                 loss="RMSE" if case["loss"] == "RMSE" else "Logloss",
                                 border_count=64, uniform_half=True)
    fp = cb.FitParams(loss=case["loss"], depth=case["depth"], iterations=case["it"], learning_rate=0.1,
                      l2_leaf_reg=3.0, score_function=case["score"], bootstrap_type=case["boot"],
                      subsample=0.7, bagging_temperature=1.0, random_seed=42,
                      boost_from_average=case["loss"] == "RMSE")
    m = cb.fit(_cols(X), borders, y, fp, staged=True)
    o = _oracle_fit(X, y, borders, fp)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.leaf_values - o.leaf_values)) <= PRED_TOL
    assert np.max(np.abs(m.staged - o.staged)) <= PRED_TOL


@pytest.mark.parametrize("score", ["SolarL2", "LOOL2", "SatL2"])
@pytest.mark.parametrize("loss,boot", [("RMSE", "No"), ("Logloss", "Bayesian")])
def test_device_fit_other_score_functions(score, loss, boot):
    # SolarL2 / LOOL2 / SatL2 (crates/cb-compute/src/score.rs:245-330): the
    # sum of per-leaf terms over the same histograms, no l2.  A level that
    # repeats one of the tree's earlier splits leaves every partition as it
    # was; all such candidates tie exactly and rounding picks among them, so
    # those levels are compared through the predictions only.
    X, y, borders = make_dataset(4000, 14, seed=17, nan_frac=0.02, loss=loss, border_count=32)
    fp = cb.FitParams(loss=loss, depth=5, iterations=5, learning_rate=0.1, l2_leaf_reg=3.0, score_function=score,
                      bootstrap_type=boot, bagging_temperature=1.0, random_seed=3,
                      boost_from_average=loss == "RMSE")
    m = cb.fit(_cols(X), borders, y, fp, staged=True)
    o = _oracle_fit(X, y, borders, fp)
    for t in range(fp.iterations):
        for l in range(fp.depth):
            a = (m.split_feature[t, l], m.split_bin[t, l])
            b = (o.split_feature[t, l], o.split_bin[t, l])
            seen_m = set(zip(m.split_feature[t, :l], m.split_bin[t, :l]))
            seen_o = set(zip(o.split_feature[t, :l], o.split_bin[t, :l]))
            assert a == b or (a in seen_m and b in seen_o), (t, l)
    assert np.max(np.abs(m.staged - o.staged)) <= PRED_TOL


def test_weighted_fit_matches_oracle():
    X, y, borders = make_dataset(6000, 16, seed=9, border_count=32)
    w = np.random.RandomState(2).choice([0.5, 1.0, 2.0, 3.0], size=X.shape[0])
    fp = cb.FitParams(loss="RMSE", depth=5, iterations=5, score_function="Cosine", bootstrap_type="Bayesian",
                      random_seed=3)
    m = cb.fit(_cols(X), borders, y, fp, weights=w, staged=True)
    o = _oracle_fit(X, y, borders, fp, weights=w)
    np.testing.assert_array_equal(m.split_feature, o.split_feature)
    np.testing.assert_array_equal(m.split_bin, o.split_bin)
    assert np.max(np.abs(m.staged - o.staged)) <= PRED_TOL


# ---- the seam's host-sample contract ----------------------------------------

def test_host_sample_path_matches_oracle_bootstrap():
    """sample_from_host=True: the caller (cb-train) draws the bootstrap on its
    host RNG and passes control ? w : 0 every tree (boosting.rs:6568-6660)."""
    X, y, borders = make_dataset(5000, 10, seed=4, border_count=32)
    n = X.shape[0]
    fp = cb.FitParams(loss="RMSE", depth=4, iterations=4, score_function="L2", bootstrap_type="Bernoulli",
                      subsample=0.7, random_seed=8)
    o = _oracle_fit(X, y, borders, fp)
    bias = cb.starting_approx(fp, y)
    rt = cb.B200Runtime()
    cfg = cb.DeviceTrainConfig(bootstrap_type="Bernoulli", sample_rate=0.7, rng_seed=8, bias=bias,
                               sample_from_host=True)
    assert rt.begin_device_training_raw("RMSE", 4, True, 1, "L2", _cols(X), borders, None, n, X.shape[1],
                                        max(len(b) for b in borders) + 1, 0.1, 3.0, cfg)
    rng = oracle.TFastRng64(8)
    approx = np.full(n, bias)
    for it in range(4):
        rng.gen_rand(); rng.gen_rand()  # PRE_TREE_DRAWS
        sw, ctl = oracle.bootstrap("Bernoulli", np.zeros(n), rng, subsample=0.7)
        sample = np.where(ctl, sw, 0.0)
        tree = rt.grow_tree_on_device(approx, y, sample)
        # replay_grow_draws + POST (device_draw_replay.rs)
        for _ in range(4):
            for _ in range(X.shape[1]):
                rng.gen_rand_real1()
            rng.gen_rand()
            for _ in range(X.shape[1]):
                rng.std_normal()
        rng.gen_rand(); rng.gen_rand()
        assert [s[0] for s in tree.splits] == list(o.split_feature[it])
        assert [s[1] for s in tree.splits] == list(o.split_bin[it])
        approx = approx + (tree.leaf_values * 0.1)[tree.leaf_of]
        assert np.max(np.abs(approx - o.staged[it])) <= PRED_TOL
    rt.end_device_training()


def test_staged_host_samples_match_oracle_bootstrap():
    """cbgpu_stage_sample: the same host-drawn samples, each staged one tree
    ahead (stage(t + 1) before grow(t), two waiting at the start), grow the
    oracle's trees; the staging rules are enforced."""
    X, y, borders = make_dataset(5000, 10, seed=4, border_count=32)
    n = X.shape[0]
    T = 5
    fp = cb.FitParams(loss="RMSE", depth=4, iterations=T, score_function="L2", bootstrap_type="Bernoulli",
                      subsample=0.7, random_seed=8)
    o = _oracle_fit(X, y, borders, fp)
    bias = cb.starting_approx(fp, y)
    rng = oracle.TFastRng64(8)
    samples = []
    for _ in range(T):
        rng.gen_rand(); rng.gen_rand()  # PRE_TREE_DRAWS
        sw, ctl = oracle.bootstrap("Bernoulli", np.zeros(n), rng, subsample=0.7)
        samples.append(np.where(ctl, sw, 0.0))
        for _ in range(4):  # replay_grow_draws + POST (device_draw_replay.rs)
            for _ in range(X.shape[1]):
                rng.gen_rand_real1()
            rng.gen_rand()
            for _ in range(X.shape[1]):
                rng.std_normal()
        rng.gen_rand(); rng.gen_rand()
    rt = cb.B200Runtime()
    cfg = cb.DeviceTrainConfig(bootstrap_type="Bernoulli", sample_rate=0.7, rng_seed=8, bias=bias,
                               sample_from_host=True)
    assert rt.begin_device_training_raw("RMSE", 4, True, 1, "L2", _cols(X), borders, None, n, X.shape[1],
                                        max(len(b) for b in borders) + 1, 0.1, 3.0, cfg)
    with pytest.raises(cb.CbGpuError, match="LengthMismatch"):
        rt.stage_sample(np.ones(n - 1))
    rt.stage_sample(samples[0])
    rt.stage_sample(samples[1])
    with pytest.raises(cb.CbGpuError, match="two staged samples"):
        rt.stage_sample(samples[2])
    with pytest.raises(cb.CbGpuError, match="staged sample"):  # a passed sample while staged ones wait
        rt.grow_tree_on_device(None, y, samples[0], resident_approx=True)
    approx = np.full(n, bias)
    for it in range(T):
        if 0 < it < T - 1:
            rt.stage_sample(samples[it + 1])
        tree = rt.grow_tree_on_device(None, y, None, resident_approx=True)
        assert [s[0] for s in tree.splits] == list(o.split_feature[it])
        assert [s[1] for s in tree.splits] == list(o.split_bin[it])
        approx = approx + (tree.leaf_values * 0.1)[tree.leaf_of]
        assert np.max(np.abs(approx - o.staged[it])) <= PRED_TOL
    with pytest.raises(cb.CbGpuError, match="no sample was passed or staged"):
        rt.grow_tree_on_device(None, y, None, resident_approx=True)
    rt.end_device_training()
    rt2 = cb.B200Runtime()
    assert rt2.begin_device_training_raw("RMSE", 4, True, 1, "L2", _cols(X), borders, None, n, X.shape[1],
                                         max(len(b) for b in borders) + 1, 0.1, 3.0, cb.DeviceTrainConfig())
    with pytest.raises(cb.CbGpuError, match="sample_from_host"):
        rt2.stage_sample(samples[0])
    rt2.end_device_training()


def test_seam_validation_errors():
    X, y, borders = make_dataset(300, 3, seed=1, border_count=8)
    nb = max(len(b) for b in borders) + 1
    rt = cb.B200Runtime()
    assert rt.begin_device_training_raw("RMSE", 3, True, 1, "L2", _cols(X), borders, None, 300, 3, nb, 0.1, 3.0,
                                        cb.DeviceTrainConfig())
    with pytest.raises(cb.CbGpuError, match="Degenerate"):
        rt.grow_tree_on_device(None, y, np.ones(300))
    with pytest.raises(cb.CbGpuError, match="LengthMismatch"):
        rt.grow_tree_on_device(np.zeros(299), y, [])
    rt.end_device_training()
    assert rt.grow_tree_on_device(None, y, []) is None  # no session: Ok(None)
    host = cb.DeviceTrainConfig(sample_from_host=True)
    assert rt.begin_device_training_raw("RMSE", 3, True, 1, "L2", _cols(X), borders, None, 300, 3, nb, 0.1, 3.0, host)
    with pytest.raises(cb.CbGpuError, match="Degenerate"):
        rt.grow_tree_on_device(None, y, [])
    with pytest.raises(cb.CbGpuError, match="LengthMismatch"):
        rt.grow_tree_on_device(None, y, np.ones(7))
    rt.end_device_training()
    # outside the covered regime: decline (Ok(false))
    for kw in (dict(depth=17), dict(plain=False), dict(score="NewtonL2"), dict(cfg=cb.DeviceTrainConfig(random_strength=1.0)),
               dict(cfg=cb.DeviceTrainConfig(grow_policy="Depthwise")), dict(cfg=cb.DeviceTrainConfig(bootstrap_type="Poisson"))):
        ok = rt.begin_device_training_raw("RMSE", kw.get("depth", 3), kw.get("plain", True), 1, kw.get("score", "L2"),
                                          _cols(X), borders, None, 300, 3, nb, 0.1, 3.0, kw.get("cfg", cb.DeviceTrainConfig()))
        assert ok is False and rt.decline_reason


def test_run_twice_bit_identical():
    X, y, borders = make_dataset(30000, 24, seed=5, nan_frac=0.05, border_count=128, loss="Logloss")
    fp = cb.FitParams(loss="Logloss", depth=7, iterations=3, score_function="Cosine", bootstrap_type="Bayesian",
                      boost_from_average=False)
    a = cb.fit(_cols(X), borders, y, fp, staged=True)
    b = cb.fit(_cols(X), borders, y, fp, staged=True)
    np.testing.assert_array_equal(a.staged, b.staged)
    np.testing.assert_array_equal(a.leaf_values, b.leaf_values)


def test_begin_u32_bins_path_matches_raw_path():
    X, y, borders = make_dataset(4000, 9, seed=6, border_count=16)
    bins = oracle.quantize(X.T.copy(), borders).astype(np.uint32)
    nb = max(len(b) for b in borders) + 1
    fp = cb.FitParams(loss="RMSE", depth=4, iterations=3, score_function="L2")
    ref = cb.fit(_cols(X), borders, y, fp, staged=True)
    rt = cb.B200Runtime()
    cfg = cb.DeviceTrainConfig(bias=ref.bias, border_counts=[len(b) for b in borders])
    lr = float(np.float32(fp.learning_rate))  # fit hands the seam the f32-narrowed rate (boosting.rs:4958)
    assert rt.begin_device_training("RMSE", 4, True, 1, "L2", bins, None, 4000, 9, nb, lr, 3.0, cfg)
    for it in range(3):
        tree = rt.grow_tree_on_device(None, y, [], resident_approx=True)
        assert [s[0] for s in tree.splits] == list(ref.split_feature[it])
        assert [s[1] for s in tree.splits] == list(ref.split_bin[it])
    np.testing.assert_array_equal(rt.resident_approx(), ref.staged[-1])
    rt.end_device_training()


def test_timing_sum_matches_per_tree_timing():
    """cbgpu_session_timing_sum adds up the per-tree figures whether or not
    each tree's timing was read in between (reads are deferred to the next
    tree's device work)."""
    X, y, borders = make_dataset(20000, 12, seed=8, border_count=32)
    nb = max(len(b) for b in borders) + 1
    per_tree, sums = [], []
    for read_each in (True, False):
        rt = cb.B200Runtime()
        cfg = cb.DeviceTrainConfig(bootstrap_type="Bayesian", rng_seed=4)
        assert rt.begin_device_training_raw("RMSE", 6, True, 1, "Cosine", _cols(X), borders, None, X.shape[0],
                                            X.shape[1], nb, 0.1, 3.0, cfg)
        rt.set_profiling(True)
        rt.timing_sum(reset=True)
        rows = []
        for _ in range(4):
            rt.grow_tree_on_device(None, y, [], leaf_of_bytes=0, resident_approx=True)
            if read_each:
                rows.append(rt.timing().copy())
        tot = rt.timing_sum()
        rt.end_device_training()
        if read_each:
            per_tree = np.array(rows)
            np.testing.assert_allclose(tot, per_tree.sum(axis=0), rtol=1e-12)
        sums.append(tot)
    # histogrammed rows and launch counts are exact and identical either way
    assert sums[0][6] == sums[1][6] == per_tree[:, 6].sum()
    assert sums[0][7] == sums[1][7]
    assert (sums[1][:6] >= 0).all() and sums[1][0] > 0 and sums[1][1] > 0


@pytest.mark.parametrize("boot", ["Bayesian", "Bernoulli", "MVS"])
def test_tree_graphs_match_direct_enqueue(boot):
    """Trees after the first replay one captured graph; enqueueing every tree
    directly must give bit-identical trees and approximants, also when the
    graph is re-captured (profiling switched on mid-fit)."""
    X, y, borders = make_dataset(30000, 16, seed=11, nan_frac=0.05, border_count=48, loss="Logloss")
    nb = max(len(b) for b in borders) + 1
    runs = []
    for graphs in (True, False):
        rt = cb.B200Runtime()
        cfg = cb.DeviceTrainConfig(bootstrap_type=boot, sample_rate=0.7, rng_seed=9)
        assert rt.begin_device_training_raw("Logloss", 6, True, 1, "Cosine", _cols(X), borders, None, X.shape[0],
                                            X.shape[1], nb, 0.1, 3.0, cfg)
        rt.set_graphs(graphs)
        trees = []
        for it in range(5):
            if it == 3:
                rt.set_profiling(True)
            t = rt.grow_tree_on_device(None, y, [], leaf_of_bytes=2, resident_approx=True)
            trees.append((t.splits, t.leaf_values.copy(), t.leaf_of.copy()))
        runs.append((trees, rt.resident_approx()))
        rt.end_device_training()
    (ta, aa), (tb, ab) = runs
    for (sa, la, oa), (sb, lb, ob) in zip(ta, tb):
        assert sa == sb
        np.testing.assert_array_equal(la, lb)
        np.testing.assert_array_equal(oa, ob)
    np.testing.assert_array_equal(aa, ab)
