"""The H2O group-sum oracle (runtime/gqa_h2o_stats.cu:41-57) pinned on the CPU:
against the reference's own H2OResidency::observe_attention (compiled from
its sources into oracle/_ref, where they exist), against the committed
fixture made from it, and against the reference CUDA test's strided,
NaN-poisoned geometry (tests/gqa_h2o_stats_tests.cu:41-79) summed in the
test's own order."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import inputs
from oracle import binding as ob

GOLDEN = Path(__file__).resolve().parent / "golden" / "h2o_vectors.npz"


def _contiguous_sums(p: np.ndarray) -> np.ndarray:
    heads, queries, keys = p.shape
    buf = inputs.h2o_layout(p, keys, queries, 4, 4 * keys, 4 * keys * queries)
    return ob.h2o_group_sums(buf, keys, queries, 4, 4 * keys, 4 * keys * queries)


def _expected_importance(seed: int, first: int, queries: int) -> np.ndarray:
    """Importance the reference policy holds after the fixture's two blocks:
    the seeded block's group sums, plus 4 * first at key 0 (the one-hot prior
    block), added in F32 as the policy does (h2o_residency.cpp:100-102)."""
    keys = first + queries
    s = _contiguous_sums(inputs.h2o_probabilities(seed, first, queries, keys))
    if first:
        s[:, 0] = np.float32(4 * first) + s[:, 0]
    return s


def test_oracle_matches_golden_fixture():
    g = np.load(GOLDEN)
    assert len(g["names"]) >= 10
    for i, (first, queries) in enumerate(g["blocks"]):
        got = _expected_importance(1000 + i, int(first), int(queries))
        assert inputs.digest(got) == str(g["importance_digest"][i]), g["names"][i]
        n = min(8, got.shape[1])
        assert np.array_equal(got[:, :n].view(np.uint32), g["importance_head"][i][:, :n].view(np.uint32))


@pytest.mark.skipif(not ob.reference_available(), reason="reference sources not built here")
@pytest.mark.parametrize("first,queries", [(0, 1), (0, 2), (0, 33), (7, 1), (40, 9), (300, 5)])
def test_oracle_matches_reference_policy(first, queries):
    """Bit-exact against the reference's CPU summation of the same block."""
    import importlib.util
    import sys

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("make_golden", mg)
    spec.loader.exec_module(mg)
    seed = 77 + first * 131 + queries
    ref = mg.h2o_reference_importance(seed, first, queries)
    got = _expected_importance(seed, first, queries)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def _reference_test_geometry(first: int):
    """tests/gqa_h2o_stats_tests.cu:41-66: ne {11, 6, 32, 1}, byte strides
    {8, 112, 704, 22528}, NaN everywhere but the valid probabilities; value
    (1 + (k + h/4) % 5) / sum over the causally available keys."""
    ne0, ne1 = 11, 6
    nb0, nb1, nb2 = 8, 112, 704
    queries = 3 if first == 0 else 2
    keys = first + queries
    p = np.zeros((32, queries, keys), dtype=np.float32)
    for h in range(32):
        for q in range(queries):
            available = first + q + 1
            den = float(sum(1 + ((k + h // 4) % 5) for k in range(available)))
            for k in range(keys):
                p[h, q, k] = np.float32((1 + ((k + h // 4) % 5)) / den) if k < available else np.float32(0)
    buf = inputs.h2o_layout(p, ne0, ne1, nb0, nb1, nb2, total_bytes=22528)
    return buf, p, keys, queries, (nb0, nb1, nb2)


@pytest.mark.parametrize("first", [0, 3])
def test_reference_strided_fixture(first):
    buf, p, keys, queries, nb = _reference_test_geometry(first)
    assert buf.nbytes == 22528  # nb[3] of the reference fixture
    got = ob.h2o_group_sums(buf, keys, queries, *nb)
    for kh in range(8):
        for k in range(keys):
            expected = np.float32(0)
            for lane in range(4):
                for q in range(queries):
                    expected = np.float32(expected + p[kh * 4 + lane, q, k])
            assert got[kh, k].view(np.uint32) == expected.view(np.uint32)
    assert np.all(np.isfinite(got))  # the NaN padding was never read


def test_order_is_head_major():
    """A case where the two summation orders differ in F32: (head, query)
    order must be kept, not (query, head)."""
    p = np.zeros((32, 2, 1), dtype=np.float32)
    p[0, 0, 0], p[0, 1, 0], p[1, 0, 0], p[1, 1, 0] = 1.0, 2.0 ** -24, -1.0, 2.0 ** -24
    got = _contiguous_sums(p)[0, 0]
    head_major = np.float32(np.float32(np.float32(np.float32(0) + p[0, 0, 0]) + p[0, 1, 0]) + p[1, 0, 0])
    head_major = np.float32(head_major + p[1, 1, 0])
    query_major = np.float32(np.float32(np.float32(np.float32(0) + p[0, 0, 0]) + p[1, 0, 0]) + p[0, 1, 0])
    query_major = np.float32(query_major + p[1, 1, 0])
    assert head_major != query_major
    assert got == head_major
