"""SolarL2 / LOOL2 / SatL2 split scores in the oracle.

The reference restates these GPU score calcers (score_calcers.cuh) in
crates/cb-compute/src/score.rs:245-330 and checks them against the same
arithmetic plus their boundary cases in
crates/cb-compute/tests/score_functions_test.rs; these tests do the same on
the reference's sample leaves: a split's score is the sequential sum of the
per-leaf terms, with no l2.
"""
import math

import numpy as np
import pytest

from oracle import oracle

LEAVES = [(4.0, 3.0), (-2.5, 5.0), (1.0, 1.5)]  # (sum of weighted ders, weight)


def _solar(s, w):
    return (-s * s) * (1.0 + 2.0 * math.log(w + 1.0)) / w if w > 1e-20 else 0.0


def _loo(s, w):
    a = w / (w - 1.0) if w > 1.0 else 0.0
    a *= a
    return a * (-s * s) / w if w > 0.0 else 0.0


def _sat(s, w):
    a = w * (w - 2.0) / (w * w - 3.0 * w + 1.0) if w > 2.0 else 0.0
    return a * (-s * s) / w if w > 0.0 else 0.0


@pytest.mark.parametrize("name,ref", [("SolarL2", _solar), ("LOOL2", _loo), ("SatL2", _sat)])
def test_terms_match_the_calcer_arithmetic(name, ref):
    for s, w in LEAVES:
        assert oracle.score_term(name, s, w) == ref(s, w)
    total = 0.0
    for s, w in LEAVES:
        total += oracle.score_term(name, s, w)
    assert abs(total - sum(ref(s, w) for s, w in LEAVES)) <= 1e-12


def test_boundaries():
    assert oracle.score_term("SolarL2", 0.0, 0.0) == 0.0
    assert oracle.score_term("LOOL2", 5.0, 1.0) == 0.0     # weight 1: adjust 0
    assert oracle.score_term("SatL2", 5.0, 2.0) == 0.0     # weight 2: adjust 0
    assert np.isfinite(oracle.score_term("SatL2", 5.0, 2.5))


def test_fit_uses_the_terms():
    # a depth-1 RMSE fit picks the border whose two children's terms sum highest
    rs = np.random.RandomState(0)
    x = rs.standard_normal(500).astype(np.float32)
    y = np.where(x > 0.3, 1.0, -1.0) + 0.1 * rs.standard_normal(500)
    borders = [np.sort(rs.standard_normal(12))]
    bins = oracle.quantize(x[None, :].copy(), borders)
    for name in ("SolarL2", "LOOL2", "SatL2"):
        fit = oracle.train(bins, [12], y, loss="RMSE", depth=1, iterations=1, score_function=name,
                           boost_from_average=False)
        der = y.copy()  # RMSE der1 at approx 0, unit weights
        best, bb = -np.inf, -1
        for b in range(12):
            left = bins[0] <= b
            sc = oracle.score_term(name, der[left].sum(), float(left.sum())) + \
                oracle.score_term(name, der[~left].sum(), float((~left).sum()))
            if sc > best + 1e-9:
                best, bb = sc, b
        assert fit.split_bin[0, 0] == bb, name
