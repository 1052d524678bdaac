"""H2O group sums on the GPU through the C-ABI (hsb_h2o_group_sums), bit for
bit against the oracle (runtime/gqa_h2o_stats.cu:41-57): key-contiguous
ggml layouts (the TMA kernel, both tile widths, one-box and multi-box
items), strided and misaligned layouts (the plain-load kernel), padding
keys and queries poisoned with NaN, the reference CUDA test's geometry, the
reference-shaped GQAH2OStatsCuda wrapper, and a full-size block checked on
sampled key windows plus the group-mass property."""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

import inputs
from oracle import binding as ob

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _run(buf: np.ndarray, ne, nb, keys: int, queries: int, offset: int = 0):
    import torch
    import hillserve_b200 as hsb

    dev = torch.from_numpy(buf).cuda()
    ptr = dev.data_ptr() + offset
    out = hsb.h2o_group_sums(ptr, ne, nb, keys, queries,
                             out=torch.full((8, keys), -7.0, dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _same(a: np.ndarray, b: np.ndarray) -> bool:
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _ggml_case(seed, first, queries, pad_keys=0, pad_queries=0):
    keys = first + queries
    p = inputs.h2o_probabilities(seed, first, queries, keys)
    ne0 = (keys + 255) // 256 * 256 + pad_keys
    ne1 = queries + pad_queries
    nb = (4, 4 * ne0, 4 * ne0 * ne1, 4 * ne0 * ne1 * 32)
    buf = inputs.h2o_layout(p, ne0, ne1, nb[0], nb[1], nb[2])
    return buf, (ne0, ne1, 32, 1), nb, keys


@pytest.mark.parametrize("first,queries,pad_keys,pad_queries", [
    (4095, 1, 0, 0),      # decode, keys a multiple of the tile
    (4095, 1, 256, 3),    # decode with padding keys and queries
    (0, 2, 0, 1), (5, 3, 0, 0), (61, 4, 0, 2),          # one box {KT, Q, 4 heads} per item
    (10, 5, 0, 0), (0, 16, 0, 0), (7, 17, 0, 5), (100, 33, 256, 0),  # {KT, 16, 1} boxes, ragged tails
    (999, 1, 0, 0), (1000, 47, 0, 1),                   # narrow tiles, ragged keys
    (9999, 1, 0, 0), (12000, 7, 0, 0), (9472, 40, 256, 2),  # wide tiles
])
def test_contiguous_layout_matches_oracle(cuda, first, queries, pad_keys, pad_queries):
    buf, ne, nb, keys = _ggml_case(31 + first + queries, first, queries, pad_keys, pad_queries)
    got = _run(buf, ne, nb, keys, queries)
    want = ob.h2o_group_sums(buf, keys, queries, nb[0], nb[1], nb[2])
    assert np.all(np.isfinite(want))
    assert _same(got, want)


@pytest.mark.parametrize("first", [0, 3])
def test_reference_test_geometry(cuda, first):
    """tests/gqa_h2o_stats_tests.cu:41-79: holes between keys (nb0 = 8),
    padding queries and keys, NaN everywhere else."""
    from test_h2o_oracle import _reference_test_geometry

    buf, p, keys, queries, nb = _reference_test_geometry(first)
    got = _run(buf, (11, 6, 32, 1), nb + (22528,), keys, queries)
    want = ob.h2o_group_sums(buf, keys, queries, *nb)
    assert _same(got, want) and np.all(np.isfinite(got))


@pytest.mark.parametrize("case", ["holes", "unaligned_rows", "unaligned_base", "head_inner"])
def test_strided_layouts_match_oracle(cuda, case):
    first, queries = 2990, 9
    keys = first + queries
    p = inputs.h2o_probabilities(5, first, queries, keys)
    offset = 0
    if case == "holes":            # two floats per key
        ne0, ne1, nb = keys, queries + 1, (8, 8 * keys + 24, (8 * keys + 24) * (queries + 1))
    elif case == "unaligned_rows":  # key-contiguous, rows not 16-byte multiples
        ne0, ne1, nb = keys + 2, queries, (4, 4 * (keys + 2), 4 * (keys + 2) * queries)
    elif case == "unaligned_base":  # aligned strides, base 4 bytes off a 16-byte boundary
        ne0, ne1, nb = 3072, queries, (4, 4 * 3072, 4 * 3072 * queries)
        offset = 4
    else:                          # [key][Q head][query] storage: heads inner to queries
        ne0, ne1, nb = keys, queries, (4, 4 * keys * 32, 4 * keys)
    core = inputs.h2o_layout(p, ne0, ne1, nb[0], nb[1], nb[2])
    buf = np.concatenate([np.full(offset, 0xFF, dtype=np.uint8), core, np.zeros(16, dtype=np.uint8)])
    got = _run(buf, (ne0, ne1, 32, 1), nb + (0,), keys, queries, offset=offset)
    want = ob.h2o_group_sums(buf, keys, queries, nb[0], nb[1], nb[2], offset=offset)
    assert _same(got, want)


def test_reduce_wrapper_like_reference(cuda):
    """GQAH2OStatsCuda.reduce: bounded buffers, timings, the sums on the host
    and the shape guards of tests/gqa_h2o_stats_tests.cu:67-95."""
    import torch
    import hillserve_b200 as hsb
    from test_h2o_oracle import _reference_test_geometry

    dev = torch.empty(22528 // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    reducer = hsb.GQAH2OStatsCuda(dev, 7)
    assert reducer.gpu_bytes() == 8 * 7 * 4 and reducer.host_bytes() == 8 * 7 * 4
    ne, nb = (11, 6, 32, 1), (8, 112, 704, 22528)
    for first in (0, 3):
        buf, p, keys, queries, _ = _reference_test_geometry(first)
        dev.copy_(torch.from_numpy(buf.view(np.float32)))
        r = reducer.reduce(dev, ne, nb, keys, queries, stream)
        assert r.elements == 8 * keys and r.d2h_bytes == 8 * keys * 4
        assert r.ready_observed_ns >= r.started_ns and r.reduction_ms >= 0 and r.d2h_ms >= 0
        want = ob.h2o_group_sums(buf, keys, queries, 8, 112, 704).reshape(-1)
        assert _same(np.asarray(r.sums), want)
    for bad_ne, k, q in (((11, 6, 8, 1), 5, 2), ((11, 6, 32, 2), 5, 2), (ne, 8, 2), (ne, 5, 7)):
        with pytest.raises(hsb.HsbError):
            reducer.reduce(dev, bad_ne, nb, k, q, stream)
    with pytest.raises(hsb.HsbError):
        reducer.reduce(dev, ne, nb, 5, 2, None)


def test_full_size_block_windows_and_mass(cuda):
    """A 512-query block over 32768 keys (2 GiB of probabilities): every
    sampled 64-key window is bit-exact against the oracle and each KV head's
    total mass is 4 x 512 (softmax rows sum to 1)."""
    import torch
    import hillserve_b200 as hsb

    keys, queries = 32768, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    probs = torch.empty((32, queries, keys), dtype=torch.float32, device="cuda")
    for h in range(32):
        logits = torch.randn((queries, keys), generator=g, device="cuda") * 3.0
        probs[h] = torch.softmax(logits, dim=1)
    nb = (4, 4 * keys, 4 * keys * queries, 4 * keys * queries * 32)
    out = hsb.h2o_group_sums(probs, (keys, queries, 32, 1), nb, keys, queries)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for k0 in (0, 4096 + 64, 20000, keys - 64):
        window = np.ascontiguousarray(probs[:, :, k0:k0 + 64].cpu().numpy())
        want = ob.h2o_group_sums(window, 64, queries, 4, 256, 256 * queries)
        assert _same(got[:, k0:k0 + 64], want), k0
    mass = got.astype(np.float64).sum(axis=1)
    assert np.all(np.abs(mass - 4 * queries) <= 1e-3 * 4 * queries)
    del probs
    torch.cuda.empty_cache()


@pytest.mark.parametrize("impl", ["b200", "ref"])
def test_reference_cuda_test_program(cuda, impl):
    """The reference's own tests/gqa_h2o_stats_tests.cu, compiled unmodified
    (oracle/Makefile) against the B200 drop-in header and libhsb_compat
    ("b200") and against the reference implementation ("ref"); both must
    pass, including its GPU-vs-CPU H2OResidency agreement checks."""
    exe = ROOT / "oracle" / "_ref" / f"gqa_h2o_stats_tests_{impl}"
    if not exe.exists():
        pytest.skip("built only where the reference sources were present")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert r.stdout.startswith("passed: CUDA real-stream F32 GQA sum")
