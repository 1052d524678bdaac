"""Cold-tier KV records (SegmentedKVStore v1) on the CPU: the oracle's FNV-1a,
record encoder and verifier and the library's host functions (file header,
extent, read plan, validation groups) against the published FNV-1a vectors,
the reference's own store, checksum and planner (compiled from its sources
into oracle/_ref where they exist) and the fixture made from them."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import inputs
from oracle import binding as ob

GOLDEN = Path(__file__).resolve().parent / "golden" / "records_vectors.npz"
HAVE_REF = ob.reference_available()


def _make_golden():
    import importlib.util
    import sys

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("make_golden", mg)
    spec.loader.exec_module(mg)
    return mg


@pytest.fixture(scope="module")
def lib():
    from hillserve_b200 import _capi

    return _capi.lib()


def test_fnv1a_published_vectors(lib):
    # FNV-1a 64-bit test vectors of the algorithm's published description.
    for text, want in ((b"", 0xCBF29CE484222325), (b"a", 0xAF63DC4C8601EC8C), (b"foobar", 0x85944171F73967E8)):
        assert ob.fnv1a64(text) == want
        buf = C.create_string_buffer(text, len(text) or 1)
        assert lib.hsb_fnv1a64(buf, len(text)) == want


def test_checksum_four_fixture():
    """The reference reader test's bytes (direct_read_batch_tests.cpp:17-19):
    the oracle's FNV-1a of every row and length equals the reference's
    four-way interleaved checksum recorded in the fixture."""
    g = np.load(GOLDEN)
    i = np.arange(4 * 65536, dtype=np.uint64)
    data = ((i // 4096 * 31 + i * 17) % 251).astype(np.uint8)
    rows = [data[j * 65536:(j + 1) * 65536] for j in range(4)]
    k = 0
    for length in (0, 1, 17, 4096, 65536):
        for n in range(1, 5):
            for j in range(n):
                assert ob.fnv1a64(rows[j][:length]) == int(g["checksum_four"][k][j])
            k += 1


@pytest.mark.parametrize("case", [0, 1, 2])
def test_segment_file_image_matches_fixture(lib, case):
    """Header (hsb_segment_header) + oracle-encoded records at the store's
    offsets reproduce, byte for byte, the file the reference store wrote."""
    mg = _make_golden()
    request, layers, positions, nbytes, payloads = mg.record_case(case)
    img = inputs.segment_image(request, layers, positions, nbytes, payloads, ob.records_encode)
    header = np.zeros(4096, dtype=np.uint8)
    assert lib.hsb_segment_header(header.ctypes.data, request, layers, positions, nbytes) == 0
    assert np.array_equal(header, img[:4096])
    assert lib.hsb_segment_extent_bytes(layers, positions, nbytes) == img.nbytes
    assert inputs.digest(img) == str(np.load(GOLDEN)[f"file{case}_digest"])


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not built here")
def test_file_image_equals_reference_store_file(tmp_path):
    mg = _make_golden()
    request, layers, positions, nbytes, payloads = mg.record_case(0)
    path = str(tmp_path / "store")
    ob.ref_segment_roundtrip(path, request, layers, positions, nbytes, 9 << 30, payloads)
    img = inputs.segment_image(request, layers, positions, nbytes, payloads, ob.records_encode)
    assert np.array_equal(np.fromfile(path, dtype=np.uint8), img)


def _store_offsets(layer, ids, positions, nbytes):
    return (4096 + (layer * positions + np.asarray(ids, dtype=np.uint64)) * (nbytes + 32)).astype(np.uint64)


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not built here")
@pytest.mark.parametrize("mutation", ["none", "payload", "position", "layer", "request", "version", "digest"])
def test_verifier_agrees_with_reference_fetch(tmp_path, mutation):
    """SegmentedKVStore::fetch (segmented_store.cpp:105-137) and the oracle
    verifier accept the same records and reject the same corruptions with
    the same kind of error."""
    request, layers, positions, nbytes = 991, 2, 48, 4096
    payloads = [inputs.record_payload(5 + l, positions, nbytes) for l in range(layers)]
    ids = np.array([3, 7, 8, 9, 20, 40, 41], dtype=np.uint64)
    target = 4096 + (1 * positions + 9) * (nbytes + 32)  # layer 1, position 9
    where = {"payload": 32 + 1000, "position": 8, "layer": 24, "request": 16, "version": 28, "digest": 0}
    off = -1 if mutation == "none" else target + where[mutation]
    path = str(tmp_path / "kv")
    ref_error = None
    try:
        got = ob.ref_segment_roundtrip(path, request, layers, positions, nbytes, 9 << 30, payloads, off, 0x40, 1,
                                       ids)
    except ob.ReferenceError_ as e:
        ref_error = str(e)
    img = np.fromfile(path, dtype=np.uint8)
    code, index, rows = ob.records_verify(img, _store_offsets(1, ids, positions, nbytes), ids, request, 1, nbytes)
    if mutation == "none":
        assert ref_error is None and code == 0
        assert np.array_equal(rows.reshape(-1), got)
        assert np.array_equal(rows, payloads[1][ids.astype(np.int64)])
    elif mutation in ("payload", "digest"):
        assert ref_error == "selected KV checksum failure" and (code, index) == (91, 3)
    else:
        assert ref_error == "on-disk identity/version mismatch" and (code, index) == (90, 3)


def test_validation_groups_order_errors(lib):
    """Identity failures precede checksum failures inside a validation group
    of four (full_gqa_runtime.cpp:394-409), record order across groups."""
    request, nbytes = 3, 256
    payload = inputs.record_payload(9, 8, nbytes)
    recs = ob.records_encode(payload, 8, nbytes, request, 0, 0)
    offsets = np.arange(8, dtype=np.uint64) * (nbytes + 32)
    ids = np.arange(8, dtype=np.uint64)
    bad = recs.copy()
    bad[1 * (nbytes + 32) + 32 + 5] ^= 1      # record 1: payload -> checksum failure
    bad[2 * (nbytes + 32) + 8] ^= 1           # record 2: position -> identity failure
    assert ob.records_verify(bad, offsets, ids, request, 0, nbytes)[:2] == (91, 1)  # fetch order
    groups = np.array([0, 0, 0, 0, 1, 1, 1, 1], dtype=np.uint32)
    assert ob.records_verify(bad, offsets, ids, request, 0, nbytes, groups=groups)[:2] == (90, 2)
    windows = (C.c_uint64 * 10)(0, 8192, 8192, 0, 3, 8192, 16384, 8192, 3, 8)
    got = np.zeros(8, dtype=np.uint32)
    assert lib.hsb_kv_read_groups(windows, 2, got.ctypes.data, 8) == 0
    assert got.tolist() == [0, 0, 0, 1, 1, 1, 1, 2]  # batches of four restart at each window
    assert lib.hsb_kv_read_groups(windows, 2, got.ctypes.data, 9) == 94  # windows do not cover the records


def _plan(lib, offsets, record_bytes, extent, window, gap, amp):
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    out = np.zeros((max(len(off), 1), 5), dtype=np.uint64)
    n = C.c_size_t(0)
    rc = lib.hsb_kv_read_plan(off.ctypes.data, len(off), record_bytes, extent, window, gap, amp, out.ctypes.data,
                              out.shape[0], C.byref(n))
    return rc, out[:n.value]


def test_read_plan_matches_fixture(lib):
    mg = _make_golden()
    g = np.load(GOLDEN)
    for seed in range(24):
        offsets, stride, extent, window, gap, amp = mg.plan_case(seed)
        rc, w = _plan(lib, offsets, stride, extent, window, gap, amp)
        assert rc == 0
        assert inputs.digest(w) == str(g["plan_digest"][seed]), seed


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not built here")
def test_read_plan_matches_reference_randomised(lib):
    rng = np.random.default_rng(2024)
    for _ in range(200):
        stride = int(rng.choice([4128, 100 + 32, 65536 + 32]))
        window = int(rng.choice([1 << 20, 65536 * 2, 262144]))
        n = int(rng.integers(0, 300))
        gaps = rng.integers(0, 3 * stride, size=n)
        offsets = (4096 + np.cumsum(stride + gaps) - stride).astype(np.uint64) if n else np.zeros(0, np.uint64)
        extent = int(((offsets[-1] + stride if n else 4096) + 4095) // 4096 * 4096) + 4096 * int(rng.integers(0, 3))
        gap, amp = int(rng.choice([0, 4096, 65536])), int(rng.integers(1000, 2001))
        rc, w = _plan(lib, offsets, stride, extent, window, gap, amp)
        assert rc == 0
        assert np.array_equal(w, ob.ref_read_plan(offsets, stride, extent, window, gap, amp))


def test_read_plan_rejections(lib):
    # kv_read_plan_tests.cpp:44-48 and the limits of kv_read_plan.hpp:22-28
    extent = 4096 * 64
    assert _plan(lib, [4096, 4096], 4128, extent, 1 << 20, 16384, 1500)[0] == 94
    assert lib.hsb_last_error() == b"unordered, overlapping or out-of-extent KV record"
    assert _plan(lib, [8192, 4096], 4128, extent, 1 << 20, 16384, 1500)[0] == 94
    assert _plan(lib, [extent - 4096], 4128, extent, 1 << 20, 16384, 1500)[0] == 94
    assert _plan(lib, [4096], 4128, extent, 2 << 20, 0, 1500)[0] == 94
    assert lib.hsb_last_error() == b"invalid bounded complete-KV read limits"
    assert _plan(lib, [4096], 4128, extent, 1 << 20, 1, 1500)[0] == 94
    assert _plan(lib, [4096], 4128, extent + 1, 1 << 20, 0, 1500)[0] == 94
    assert lib.hsb_last_error() == b"invalid complete-KV record geometry"
    assert _plan(lib, [], 4128, extent, 1 << 20, 0, 1500) [0] == 0


def test_segment_geometry_bounds(lib):
    # segmented_store.cpp:25
    h = np.zeros(4096, dtype=np.uint8)
    assert lib.hsb_segment_header(h.ctypes.data, 1, 0, 10, 4096) == 93
    assert lib.hsb_segment_header(h.ctypes.data, 1, 129, 10, 4096) == 93
    assert lib.hsb_segment_header(h.ctypes.data, 1, 1, 66049, 4096) == 93
    assert lib.hsb_segment_header(h.ctypes.data, 1, 1, 10, 65537) == 93
    assert lib.hsb_segment_extent_bytes(32, 66048, 4096) == (4096 + 32 * 66048 * 4128 + 4095) // 4096 * 4096
    assert lib.hsb_segment_extent_bytes(0, 1, 1) == 0
    p = C.c_void_p(0x1000)
    st = C.c_void_p(0x2000)
    assert lib.hsb_kv_records_encode(p, 4096, 0, 4096, 1, 0, 0, p, None) == 1  # empty append
    assert lib.hsb_kv_records_encode(p, 4095, 1, 4096, 1, 0, 0, p, None) == 1
    assert lib.hsb_kv_records_encode(p, 65537, 1, 65537, 1, 0, 0, p, None) == 93
    assert lib.hsb_kv_records_verify(p, 0, p, p, None, 0, 1, 0, 4096, p, 4096, None, 0, st, None) == 0  # nothing
    assert lib.hsb_kv_records_verify(p, 0, p, p, None, 1, 1, 0, 4096, p, 4095, None, 0, st, None) == 1
