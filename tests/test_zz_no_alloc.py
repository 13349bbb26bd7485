"""The allocation-free histogram entry point, checked against the regular one.

cbgpu_histogram_noalloc is for callers that cannot allocate device memory
when they need a histogram (for example code under CUDA graph capture, or a
process whose device memory belongs to its own pool allocator).  It must give
the same histogram as cbgpu_histogram, call after call, although every call
reuses one fixed scratch array that keeps the previous call's contents.

This file is named to be collected last: a failure here leaves every other
test already run.  It passes alone in a fresh process (the first call sets up
the scratch address) and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HIST_RTOL = 1e-6  # the histogram bar used by the parity tests


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _case(n, F, B, seed):
    rs = np.random.RandomState(seed)
    bins = rs.randint(0, B, size=(n, F)).astype(np.uint8)
    if n > 10:
        bins[: n // 7, 0] = 0  # a hot bin
    g = rs.standard_normal(n) * rs.exponential(1.0, n)
    h = rs.exponential(1.0, n)
    return bins, g, h


def _noalloc(torch, bins, g, h, B):
    import catboost_rs_b200 as cb
    L = cb.load_library()
    n, F = bins.shape
    stride = (F + 31) // 32 * 32
    dev = torch.device("cuda", 0)
    d_bins = torch.zeros((max(n, 1), stride), dtype=torch.uint8, device=dev)
    d_bins[:n, :F] = torch.from_numpy(bins).to(dev)
    d_g = torch.from_numpy(g).to(dev)
    d_h = torch.from_numpy(h).to(dev)
    d_out = torch.full((F, B, 2), float("nan"), dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)
    rc = L.cbgpu_histogram_noalloc(C.c_void_p(d_bins.data_ptr()), n, F, stride, B,
                                   C.c_void_p(d_g.data_ptr()), C.c_void_p(d_h.data_ptr()),
                                   C.c_void_p(d_out.data_ptr()), C.c_void_p(stream.cuda_stream))
    assert rc == 0, L.cbgpu_last_error().decode()
    stream.synchronize()
    return d_out.cpu().numpy()


def test_noalloc_histogram_matches_cbgpu_histogram_twice(torch_cuda):
    import catboost_rs_b200 as cb
    # two calls in a row on different inputs and shapes: the second must not
    # see anything the first one left in the shared scratch
    for n, F, B, seed in ((50_000, 40, 129, 1), (20_001, 9, 17, 2)):
        bins, g, h = _case(n, F, B, seed)
        got = _noalloc(torch_cuda, bins, g, h, B)
        ref = cb.histogram(bins, g, h, None, 1, B)[0]
        assert got.shape == ref.shape
        scale = np.abs(ref) + 1e-300
        assert np.all(np.abs(got - ref) <= HIST_RTOL * scale + 1e-12)


def test_noalloc_rejects_sizes_beyond_its_limit(torch_cuda):
    import catboost_rs_b200 as cb
    L = cb.load_library()
    rc = L.cbgpu_histogram_noalloc(None, 262145, 4, 32, 8, None, None, None, None)
    assert rc == 2
    assert "262144" in L.cbgpu_last_error().decode()
    rc = L.cbgpu_histogram_noalloc(None, 10, 300, 320, 256, None, None, None, None)
    assert rc == 2
