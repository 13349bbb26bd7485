"""Pin the oracle's border selection to upstream CatBoost 1.2.10's border sets.

The fixtures (tests/golden/borders.npz, extracted by make_golden.py from the
reference's crates/cb-oracle/fixtures/{border_types,borders_quant}) are the
standalone Pool.quantize().save_quantization_borders() output for five small
corpora, every border type and several budgets.  The reference's own tests
(crates/cb-data/tests/border_types_oracle_test.rs, borders_quant_oracle_test.rs)
compare its binarizers against the same sets.  Upstream writes the borders as
text with ~10 significant digits, which identifies an f32 uniquely, so the bar
is exact equality of the f32 values (stricter than the reference's own 1e-5
comparison, crates/cb-oracle/src/compare.rs:46-148).
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "borders.npz")
# The exact dynamic-programming binarizers are not restated (no path here uses them).
RESTATED = {"GreedyLogSum", "GreedyMinEntropy", "Median", "Uniform", "UniformAndQuantiles"}


def _cells():
    z = np.load(GOLDEN)
    return z, json.loads(str(z["cells"]))


def _cell_ids():
    _, cells = _cells()
    return [c["stem"] for c in cells if c["border_type"] in RESTATED]


@pytest.mark.parametrize("stem", _cell_ids())
def test_borders_match_upstream(stem):
    z, cells = _cells()
    c = next(c for c in cells if c["stem"] == stem)
    X = z[f"X__{c['dataset']}"]
    flat, counts = z[f"B__{stem}"], z[f"C__{stem}"]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    assert X.shape[1] == counts.size
    for f in range(X.shape[1]):
        got = oracle.select_borders(X[:, f], c["border_count"], c["border_type"], c["nan_mode"])
        want = flat[offs[f]:offs[f + 1]]
        assert got.size == want.size, (f, got.size, want.size)
        # every selected border is an f32 value widened to f64
        assert np.array_equal(got.astype(np.float32).astype(np.float64), got)
        g32, w32 = got.astype(np.float32), want.astype(np.float32)
        assert np.array_equal(g32, w32), (f, np.flatnonzero(g32 != w32)[:5])


def test_every_restated_type_is_pinned():
    _, cells = _cells()
    covered = {c["border_type"] for c in cells}
    assert RESTATED <= covered
    assert sum(c["border_type"] in RESTATED for c in cells) >= 40


def test_nan_sentinels():
    rs = np.random.RandomState(3)
    col = rs.standard_normal(5000).astype(np.float32)
    col[::17] = np.nan
    lo = oracle.select_borders(col, 16, "GreedyLogSum", "Min")
    hi = oracle.select_borders(col, 16, "GreedyLogSum", "Max")
    fmax = float(np.finfo(np.float32).max)
    # the sentinel spends one slot of the budget either way
    assert lo.size == 16 and lo[0] == -fmax
    assert hi.size == 16 and hi[-1] == fmax
    assert np.array_equal(lo[1:], hi[:-1])
    with pytest.raises(ValueError):
        oracle.select_borders(col, 16, "GreedyLogSum", "Forbidden")
    clean = oracle.select_borders(col[~np.isnan(col)], 16, "GreedyLogSum", "Min")
    assert clean.size == 16 and clean[0] != -fmax


def test_sample_indices_over_the_cap():
    # borders.rs:504-520: a fixed-seed 200k sample, sorted, depending only on n
    a = oracle.border_sample_indices(250_000)
    b = oracle.border_sample_indices(250_000)
    assert a.size == 200_000 and np.array_equal(a, b)
    assert np.all(np.diff(a) > 0) and a[0] >= 0 and a[-1] < 250_000
    assert np.array_equal(oracle.border_sample_indices(1000), np.arange(1000))
    # a column over the cap selects from exactly the sampled rows
    rs = np.random.RandomState(5)
    col = rs.standard_normal(250_000).astype(np.float32)
    got = oracle.select_borders(col, 32, "GreedyLogSum", "Min")
    want = oracle.select_borders(col[a], 32, "GreedyLogSum", "Min")
    assert np.array_equal(got, want)


def test_degenerate_columns():
    assert oracle.select_borders(np.zeros(0, np.float32), 8).size == 0
    assert oracle.select_borders(np.ones(100, np.float32), 8).size == 0
    assert oracle.select_borders(np.array([1.0], np.float32), 8).size == 0
    two = oracle.select_borders(np.array([1.0, 2.0], np.float32), 8)
    assert np.array_equal(two, [1.5])
    # a border of zero is emitted as +0.0 whichever signed zeros straddle it
    z = oracle.select_borders(np.array([-0.0, -0.0, 0.0, 0.0, 1.0, 1.0], np.float32), 2, "Median")
    assert z.size >= 1 and np.all(z[z == 0] == 0) and not np.any(np.signbit(z[z == 0]))
