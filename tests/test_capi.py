"""The C-ABI library loads and exports every entry point include/hsb.h
declares; host-side argument validation follows the reference's checks and
wording.  CPU only: every call here is rejected before any CUDA work."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_functions() -> set[str]:
    text = (ROOT / "include" / "hsb.h").read_text()
    return set(re.findall(r"^\s*(?:const\s+)?[\w]+\s*\*?\s*(hsb_\w+)\s*\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib():
    from hillserve_b200 import _capi

    if not _capi.LIB_PATH.exists():
        from hillserve_b200 import build

        build.build()
    return _capi.lib()


def test_exports_every_declared_symbol(lib):
    from hillserve_b200 import _capi

    declared = header_functions()
    assert len(declared) >= 29
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_capi.declared_symbols())
    assert lib.hsb_abi_version() == 1


def test_v3_pipeline_rejects_invalid_counts_without_access(lib):
    # kernel_check.cpp:116-121: invalid N never touches memory (null pointers).
    for n in (0, 1, 32, 63, 65, 32769, 0xFFFFFFFF):
        assert lib.hsb_score_pipeline_v3(None, None, n, None, None) == 12
        assert "requires64<=N<=32768" in lib.hsb_last_error().decode()


def test_score_argument_checks(lib):
    from hillserve_b200._capi import KeyView

    q = C.c_void_p(0x1000)
    views = (KeyView * 1)(KeyView(None, 1, 1024))
    assert lib.hsb_score_views(q, views, 1, C.c_void_p(0x2000), None) == 10
    assert lib.hsb_last_error() == b"full GQA CPU key view shape/stride/extent"
    views[0] = KeyView(0x3000, 0, 1024)
    assert lib.hsb_score_views(q, views, 1, C.c_void_p(0x2000), None) == 10
    views[0] = KeyView(0x3000, 1, 1)
    assert lib.hsb_score_views(q, views, 1, C.c_void_p(0x2000), None) == 10
    views[0] = KeyView(0x3000, 2**62, 1024)
    assert lib.hsb_score_views(q, views, 1, C.c_void_p(0x2000), None) == 10
    assert lib.hsb_score_views(q, views, 0, C.c_void_p(0x2000), None) == 10
    assert lib.hsb_last_error() == b"full GQA CPU query/views shape"
    views[0] = KeyView(0x3000, 1, 1024)
    assert lib.hsb_score_views(q, views, 1, q, None) == 11
    assert lib.hsb_last_error() == b"full GQA CPU output must not alias the query"


def test_select_argument_checks(lib):
    ws = C.c_void_p(0x10000)
    p = C.c_void_p(0x1000)

    def sel(heads, stride, valid, alpha, ratio, kcap=100):
        return lib.hsb_select(p, 0, heads, stride, valid, C.c_float(alpha), C.c_float(ratio), 0, p, kcap, p,
                              C.c_void_p(0x2000), ws, 1 << 30, None)

    for args in ((0, 8, 4, 1.0, 0.2), (129, 8, 4, 1.0, 0.2), (2, 8, 0, 1.0, 0.2), (2, 4, 8, 1.0, 0.2)):
        assert sel(*args) == 20
        assert lib.hsb_last_error() == b"GQA selector shape"
    for args in ((2, 8, 4, -1.0, 0.2), (2, 8, 4, float("nan"), 0.2), (2, 8, 4, float("inf"), 0.2),
                 (2, 8, 4, 1.0, 0.0), (2, 8, 4, 1.0, 1.5), (2, 8, 4, 1.0, float("nan"))):
        assert sel(*args) == 21
        assert lib.hsb_last_error() == b"GQA selector numeric parameters"
    # the ID buffer must hold min(floor(valid*ratio), valid) per head
    assert sel(32, 4096, 4096, 1.0, 0.2, kcap=818) == 28


def test_union_and_pack_shape_checks(lib):
    p = C.c_void_p(0x1000)
    assert lib.hsb_union(p, 4, p, 1, 0, p, p, None, p, 1 << 20, None) == 30
    assert lib.hsb_union(p, 4, p, 1, 66049, p, p, None, p, 1 << 20, None) == 30
    assert lib.hsb_last_error() == b"GQA union bounds"

    def pack(npos, last, count, nphys, payload_bytes):
        return lib.hsb_pack(p, 4, p, 1, p, npos, last, p, nphys, p, payload_bytes, count, p, p, None, None, p,
                            1 << 24, None)

    for args in ((0, 10, 32, 1, 4096), (257, 10, 32, 1, 4096), (1, 66048, 32, 1, 4096), (1, 10, 0, 1, 4096),
                 (1, 10, 66049, 1, 4096), (1, 10, 32, 2, 4096)):
        assert pack(*args) == 40
        assert lib.hsb_last_error() == b"GQA packing shape"


def test_cover_range_checks(lib):
    p = C.c_void_p(0x1000)
    # position 0, position >= capacity, and cap == 0 are rejected
    assert lib.hsb_prefetch_cover(p, 192, 0, C.c_float(5.0), 0, p, 0, p, p, 1 << 24, None) == 60
    assert lib.hsb_prefetch_cover(p, 192, 192, C.c_float(5.0), 0, p, 38, p, p, 1 << 24, None) == 60
    assert lib.hsb_prefetch_cover(p, 192, 3, C.c_float(5.0), 0, p, 0, p, p, 1 << 24, None) == 60


def test_compat_handles_exported():
    """Every C handle include/hsb_compat.h declares is exported by libhsb_compat."""
    from hillserve_b200 import build

    text = (ROOT / "include" / "hsb_compat.h").read_text()
    names = set(re.findall(r"(hsb_compat_\w+)\s*\(", text))
    assert len(names) == 3
    compat = C.CDLL(str(build.COMPAT_LIB))
    for name in names:
        assert hasattr(compat, name), name


def test_h2o_shape_guards(lib):
    """runtime/gqa_h2o_stats.cu:110-133 and the guards of
    tests/gqa_h2o_stats_tests.cu:90-95, rejected before any device work."""
    p = C.c_void_p(0x1000)
    ne = (C.c_int64 * 4)(11, 6, 32, 1)
    nb = (C.c_size_t * 4)(8, 112, 704, 22528)

    def call(ne_, nb_, keys, queries, cap=7, probs=p):
        return lib.hsb_h2o_group_sums(probs, ne_, nb_, keys, queries, p, cap, None, None)

    bad_heads = (C.c_int64 * 4)(11, 6, 8, 1)
    assert call(bad_heads, nb, 5, 2) == 81
    assert lib.hsb_last_error() == b"H2O reduction requires [keys,queries,32,1] actual attention"
    bad_streams = (C.c_int64 * 4)(11, 6, 32, 2)
    assert call(bad_streams, nb, 5, 2) == 81
    assert call(ne, nb, 8, 2) == 80  # capacity overrun
    assert lib.hsb_last_error() == b"H2O reduction invalid pointer, actual CUDA stream or capacity"
    assert call(ne, nb, 5, 7) == 81  # padding query overrun
    assert call(ne, nb, 12, 2, cap=12) == 81  # key overrun
    assert call(ne, nb, 0, 2) == 80 and call(ne, nb, 5, 0) == 80
    assert call(ne, nb, 5, 2, probs=None) == 80
    assert call(ne, (C.c_size_t * 4)(2, 112, 704, 0), 5, 2) == 82
    assert call(ne, (C.c_size_t * 4)(8, 110, 704, 0), 5, 2) == 82
    assert lib.hsb_last_error() == b"H2O reduction invalid F32 tensor stride"
    assert call(ne, nb, 5, 2, probs=C.c_void_p(0x1002)) == 84
    assert lib.hsb_last_error() == b"H2O reduction requires aligned F32 tensor"
    huge = (C.c_size_t * 4)(1 << 62, 112, 704, 0)
    assert call(ne, huge, 5, 2) == 83
    assert lib.hsb_status_message(84) == b"H2O reduction requires aligned F32 tensor"


def test_status_messages_match_reference_wording(lib):
    want = {
        22: b"nonfinite head0 score", 23: b"F16 threshold overflow", 24: b"nonfinite GQA score",
        26: b"public F16 count overflow; long-count policy extension required",
        27: b"public F16 mean overflow; long-count policy extension required",
        31: b"GQA duplicate/future selected ID", 41: b"duplicate/future physical position",
        42: b"per-head selection exceeds slots", 43: b"future or missing selected KV",
        70: b"full GQA zero selection; no dense/current-token fallback",
    }
    for code, msg in want.items():
        assert lib.hsb_status_message(code) == msg


def test_workspace_queries_are_pure(lib):
    assert lib.hsb_select_workspace_bytes(32, 32768, 32768, 6553) >= 32 * 2 * 6553 * 8
    assert lib.hsb_union_workspace_bytes(32768) >= 32768 * 4
    assert lib.hsb_attention_workspace_bytes(6553) > 0
    assert lib.hsb_layer_workspace_bytes(32768, 6553) >= lib.hsb_select_workspace_bytes(32, 32768, 32768, 6553)


def test_ctypes_byref_is_accepted_for_pointer_arguments():
    x = C.c_uint32(0)
    assert C.c_void_p.from_param(C.byref(x)) is not None


def test_python_mirror_refuses_pageable_host_tensors():
    """A kernel given a pageable host address faults the GPU; the Python
    mirror refuses such a tensor before any call reaches the library."""
    torch = pytest.importorskip("torch")
    import hillserve_b200 as hsb

    q = torch.zeros(4096, dtype=torch.int16)  # pageable host memory
    with pytest.raises(hsb.InvalidArgument, match="pageable host tensor"):
        hsb.score_pipeline_v3(q, q, 64, out=q)
    assert hsb._ptr(None).value is None
