"""The allocation-free histogram entry point, checked against the CPU oracle.

cbgpu_histogram_noalloc is for callers that cannot allocate device memory
when they need a histogram (a process whose device memory belongs to its own
pool allocator, a host framework that forbids allocation on its hot path).
Every call reuses one fixed scratch array that keeps the previous call's
contents, so the checks run two calls in a row on different inputs and
shapes, and each result must match the oracle's f64 histogram
(oracle/cb_oracle.c orc_build_histogram, histogram.rs:643-717) within the
parity tests' bar: 1e-6 of the sum of |contribution| per cell.

This file is named to be collected last: a failure here leaves every other
test already run.  It passes alone in a fresh process (the first call sets up
the scratch address) and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

HIST_RTOL = 1e-6  # the histogram bar of the parity tests (test_gpu_parity.py)
CBGPU_ERR_INVALID = 2
CBGPU_ERR_DEVICE = 6


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _case(n, F, B, seed, g_scale=1.0):
    rs = np.random.RandomState(seed)
    bins = rs.randint(0, B, size=(n, F)).astype(np.uint8)
    if n > 10:
        bins[: n // 7, 0] = 0  # a hot bin
    g = rs.standard_normal(n) * rs.exponential(1.0, n) * g_scale
    h = rs.exponential(1.0, n)
    return bins, g, h


def _noalloc(torch, bins, g, h, B, expect=0):
    import catboost_rs_b200 as cb
    L = cb.load_library()
    n, F = bins.shape
    stride = (F + 31) // 32 * 32
    dev = torch.device("cuda", 0)
    d_bins = torch.zeros((max(n, 1), stride), dtype=torch.uint8, device=dev)
    d_bins[:n, :F] = torch.from_numpy(bins).to(dev)
    d_g = torch.from_numpy(g).to(dev)
    d_h = torch.from_numpy(h).to(dev)
    d_out = torch.full((F, B, 2), 7.0, dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)
    rc = L.cbgpu_histogram_noalloc(C.c_void_p(d_bins.data_ptr()), n, F, stride, B,
                                   C.c_void_p(d_g.data_ptr()), C.c_void_p(d_h.data_ptr()),
                                   C.c_void_p(d_out.data_ptr()), C.c_void_p(stream.cuda_stream))
    assert rc == expect, L.cbgpu_last_error().decode()
    stream.synchronize()
    return d_out.cpu().numpy()


def _check_against_oracle(got, bins, g, h, B):
    ref = oracle.build_histogram(bins.T.copy(), g, h, None, 1, B)[0]
    mag = oracle.build_histogram(bins.T.copy(), np.abs(g), np.abs(h), None, 1, B)[0]
    assert got.shape == ref.shape
    assert np.all(np.abs(got - ref) <= HIST_RTOL * mag + 1e-300)


def test_noalloc_histogram_matches_oracle_twice(torch_cuda):
    # two calls in a row on different inputs and shapes: the second must not
    # see anything the first one left in the shared scratch
    for n, F, B, seed in ((50_000, 40, 129, 1), (20_001, 9, 17, 2)):
        bins, g, h = _case(n, F, B, seed)
        _check_against_oracle(_noalloc(torch_cuda, bins, g, h, B), bins, g, h, B)


def test_noalloc_histogram_tiny_and_huge_magnitudes(torch_cuda):
    # the fixed-point scale follows any finite magnitude (max |g| near 1e-300
    # needs a 2^1030 scale, max |g| near 1e300 a 2^-963 one)
    for scale, seed in ((1e-300, 3), (1e300, 4)):
        bins, g, h = _case(30_000, 12, 64, seed, g_scale=scale)
        _check_against_oracle(_noalloc(torch_cuda, bins, g, h, 64), bins, g, h, 64)


def test_noalloc_rejects_non_finite_g_or_h(torch_cuda):
    bins, g, h = _case(5_000, 8, 32, 5)
    g[1234] = np.nan
    got = _noalloc(torch_cuda, bins, g, h, 32, expect=CBGPU_ERR_DEVICE)
    assert np.isnan(got).all()  # no histogram was built
    bins, g, h = _case(5_000, 8, 32, 6)
    h[17] = np.inf
    _noalloc(torch_cuda, bins, g, h, 32, expect=CBGPU_ERR_DEVICE)
    # the error word is cleared by the next call
    bins, g, h = _case(7_000, 8, 32, 7)
    _check_against_oracle(_noalloc(torch_cuda, bins, g, h, 32), bins, g, h, 32)


def test_noalloc_rejects_sizes_beyond_its_limit(torch_cuda):
    import catboost_rs_b200 as cb
    L = cb.load_library()
    rc = L.cbgpu_histogram_noalloc(None, 262145, 4, 32, 8, None, None, None, None)
    assert rc == CBGPU_ERR_INVALID
    assert "262144" in L.cbgpu_last_error().decode()
    rc = L.cbgpu_histogram_noalloc(None, 10, 300, 320, 256, None, None, None, None)
    assert rc == CBGPU_ERR_INVALID
