"""Stage 1 parity on the GPU: the sm_100a scorer against the oracle and the
reference's golden outputs, bit-exact, through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from conftest import dev_u16, host_u16
from test_oracle_pin import _pipeline_markers

pytestmark = pytest.mark.gpu


def gpu_score(hsb, q, data, n, stride):
    import torch

    out = hsb.score_full_gqa(dev_u16(q), [(dev_u16(data), n, stride)])
    torch.cuda.synchronize()
    return host_u16(out)


def test_reference_test_vectors(cuda, golden):
    import torch

    g = golden("scorer_vectors.npz")
    want = dict(zip(g["names"].tolist(), g["score_digest"].tolist()))
    rng = inputs.XorShift32(0x7F123451)
    for n in (1, 2, 7, 8, 9, 17, 65, 129):
        for stride in (1024, 2048):
            q, data = inputs.cpu_test_case(rng, n, stride)
            qd, kd = dev_u16(q), dev_u16(data)
            s = cuda.score_full_gqa(qd, [(kd, n, stride)])
            assert inputs.digest(host_u16(s)) == want[f"n{n}_s{stride}"], (n, stride)
            # second call with the query's sign flipped reuses the scorer (full_gqa_cpu_tests.cpp:56-60)
            q2 = q ^ np.uint16(0x8000)
            s2 = cuda.score_full_gqa(dev_u16(q2), [(kd, n, stride)])
            torch.cuda.synchronize()
            from oracle import binding as ob

            assert np.array_equal(host_u16(s2), ob.score(q2, data, n, stride))
            if n >= 9:
                views = [(kd[7 * stride:], 2, stride), (kd, 3, stride), (kd[stride:], 1, stride)]
                mv = cuda.score_full_gqa(qd, views)
                assert inputs.digest(host_u16(mv)) == want[f"n{n}_s{stride}_views"]


def test_kernel_check_markers_and_cancellation(cuda, ob):
    n = 192
    q, k = _pipeline_markers(n)
    s = gpu_score(cuda, q, k, n, 1024)
    t = np.arange(n)
    assert np.array_equal(s[0], (t + 1).astype(np.uint16))
    assert np.array_equal(s[28], (0x8000 | (t + 1)).astype(np.uint16))
    assert np.all(s[31] == 0)
    assert np.array_equal(s, ob.score(q, k, n, 1024))
    # kernel_check.cpp:133-142: cancellation/order witness with edge values.
    edge = [0, 0x8000, 1, 0x8001, 0x3FF, 0x400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF]
    q = np.zeros(4096, dtype=np.uint16)
    kk = np.zeros(n * 1024, dtype=np.uint16)
    for h in range(32):
        q[h * 128:h * 128 + 3] = [0x6C00, 0x3C00, 0xEC00]
        for c in range(3, 128):
            q[h * 128 + c] = edge[(h + c) % 10]
    for tt in range(n):
        for h in range(8):
            base = (tt * 8 + h) * 128
            kk[base:base + 3] = [0x6C00, 0x3C00, 0x6C00]
            kk[base + 3:base + 128] = [(tt + h + c) % 1024 for c in range(3, 128)]
    assert np.array_equal(gpu_score(cuda, q, kk, n, 1024), ob.score(q, kk, n, 1024))


def test_edge_fills(cuda, ob):
    n = 9
    for qv, kv in ((1, 1), (None, 0x7BFF), (0x7BFF, 0x7BFF), (0x8000, 0x7BFF)):
        q = np.where(np.arange(4096) % 2, 0xFBFF, 0x7BFF).astype(np.uint16) if qv is None else \
            np.full(4096, qv, dtype=np.uint16)
        data = np.full(n * 1024, kv, dtype=np.uint16)
        assert np.array_equal(gpu_score(cuda, q, data, n, 1024), ob.score(q, data, n, 1024))


@pytest.mark.parametrize("n", [64, 128, 192, 256, 320, 1024])
def test_random_pipeline_values(cuda, ob, n):
    rng = inputs.XorShift32(0x62C83E17 + n)
    q = np.array([inputs.pipeline_sample(rng) for _ in range(4096)], dtype=np.uint16)
    k = np.random.default_rng(n).integers(0, 1 << 16, n * 1024, dtype=np.uint32).astype(np.uint16)
    k = (k & 0x83FF) | ((k >> 10) % 17 << 10).astype(np.uint16)
    assert np.array_equal(gpu_score(cuda, q, k, n, 1024), ob.score(q, k, n, 1024))


@pytest.mark.parametrize("n", [1, 31, 33, 100, 1000])
def test_ragged_and_interleaved(cuda, ob, n):
    q, k, _ = inputs.config1(n, seed=7)
    v = inputs.values(7, n)
    rows = inputs.interleave(k, v, n)
    assert np.array_equal(gpu_score(cuda, q, k, n, 1024), ob.score(q, k, n, 1024))
    assert np.array_equal(gpu_score(cuda, q, rows, n, 2048), ob.score(q, rows, n, 2048))


@pytest.mark.parametrize("n", [64, 1024, 4096, 16384])
def test_config1_golden(cuda, golden, n):
    g = golden(f"config1_n{n}.npz")
    q, k, _ = inputs.config1(n, seed=0)
    assert inputs.digest(q, k) == g["input_digest"]
    s = gpu_score(cuda, q, k, n, 1024)
    assert inputs.digest(s) == g["raw_digest"]


def test_max_shape_32768(cuda, ob):
    """kernel_check.cpp:143-144 max shape, against the oracle."""
    n = 32768
    q, k, _ = inputs.config1(n, seed=3)
    assert np.array_equal(gpu_score(cuda, q, k, n, 1024), ob.score(q, k, n, 1024, threads=8))


def test_v3_pipeline_contract(cuda, ob):
    import torch

    sentinel = torch.full((32, 64), 0x1234, dtype=torch.int16, device="cuda")
    q = torch.zeros(4096, dtype=torch.int16, device="cuda")
    for n in (0, 1, 32, 63, 65, 32769):
        with pytest.raises(cuda.InvalidArgument):
            cuda.score_pipeline_v3(q, q, n, out=sentinel)
    assert bool((sentinel == 0x1234).all())
    qn, kn, _ = inputs.config1(192, seed=5)
    s = cuda.score_pipeline_v3(dev_u16(qn), dev_u16(kn), 192)
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(s), ob.score(qn, kn, 192, 1024))


def test_scale_exhaustive(cuda, ob):
    """The runtime's F16 / sqrtf(128) on every binary16 value."""
    import torch

    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = cuda.scale_scores(dev_u16(allbits))
    torch.cuda.synchronize()
    got = host_u16(out)
    want = ob.scale(allbits)
    finite = (allbits & 0x7C00) != 0x7C00
    assert np.array_equal(got[finite], want[finite])
    assert np.array_equal(got[~finite] & 0x7C00, want[~finite] & 0x7C00)
