"""The C-ABI library loads and exports every entry point include/cbgpu.h declares.

No compute calls: this runs on the CPU-only build container.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cbgpu.h")
LIB = os.path.join(ROOT, "catboost_rs_b200", "libcbgpu.so")


def declared_symbols():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"CBGPU_API\s+[\w\s\*]+?\b(cbgpu_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from catboost_rs_b200 import build
        build.build()
    return ctypes.CDLL(LIB)


def test_header_declares_the_seam():
    syms = declared_symbols()
    for s in ("cbgpu_begin", "cbgpu_begin_raw", "cbgpu_grow_tree", "cbgpu_end",
              "cbgpu_compute_gradients", "cbgpu_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    from catboost_rs_b200 import _lib
    assert sorted(_lib.EXPORTS) == declared_symbols()


def test_version_string(lib):
    lib.cbgpu_version.restype = ctypes.c_char_p
    assert lib.cbgpu_version().startswith(b"cbgpu")


def test_begin_args_layout_matches_header():
    # the ctypes mirror of cbgpu_begin_args must list the header's fields in order
    from catboost_rs_b200._lib import BeginArgs
    with open(HEADER) as f:
        text = f.read()
    body = text[text.index("typedef struct {", text.index("cbgpu_grow_policy")):text.index("} cbgpu_begin_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = re.findall(r"\b(\w+);", body)
    assert [f for f, _ in BeginArgs._fields_] == fields


def test_loss_ids_match_the_header():
    # every cbgpu_loss enumerator and the host map agree, so a new loss id
    # cannot drift between include/cbgpu.h and the Python mirror
    from catboost_rs_b200 import runtime
    hdr = open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "include", "cbgpu.h")).read()
    body = hdr[hdr.index("CBGPU_LOSS_RMSE = 0"):hdr.index("} cbgpu_loss;")]
    ids = {k: int(v) for k, v in re.findall(r"CBGPU_LOSS_(\w+)\s*=\s*(\d+)", body)}
    norm = lambda s: s.upper().replace("_", "")  # noqa: E731
    by_name = {norm(k): v for k, v in ids.items()}
    for name, v in runtime.LOSS.items():
        assert by_name.get(norm(name)) == v, name
    assert set(ids.values()) <= set(runtime.LOSS.values())


def test_staging_rejects_a_null_session_on_the_host(lib):
    # argument checks run before any CUDA call
    lib.cbgpu_stage_sample.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    lib.cbgpu_stage_sample.restype = ctypes.c_int
    lib.cbgpu_last_error.restype = ctypes.c_char_p
    assert lib.cbgpu_stage_sample(None, None, 0) == 2  # CBGPU_ERR_INVALID
    assert b"null session" in lib.cbgpu_last_error()
