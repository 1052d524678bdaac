"""The attention and rehearsal restatements of the oracle against an
independent numpy statement of the same mathematics.

The reference runs stage 4 (softmax(K.q / sqrt(128) + mask) . V per query
head, runtime/gqa_delivery.cpp:19-20) and the rehearsal query (W x, then
NORM-mode RoPE, patches/llama-b6000-round2.patch:303-317) in ggml, which is
not part of the reference tree, so the oracle's double-precision C
restatements are what the GPU is checked against.  Here each is checked
against numpy on the layouts the library uses: the packed delivery layout
(K [slot][32][128], V [32][128][slot], mask [32][qpad][slot], query row 0),
the compact live-slot layout (per-head lengths), the token-major dense cache
(query head h reads KV head h / 4), and the float ports timed as the CPU
baseline.  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

H, D = 32, 128
SCALE = float(np.float32(1.0) / np.sqrt(np.float32(128.0)))  # 1/sqrt(128) rounded to F32, as the graph's scale


def _f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def _softmax(x):
    m = np.max(x, axis=-1, keepdims=True)
    ok = np.isfinite(m)
    e = np.where(ok, np.exp(x - np.where(ok, m, 0.0)), 0.0)  # a row with no live slot gives zeros
    s = e.sum(axis=-1, keepdims=True)
    return np.where(s > 0, e / np.where(s > 0, s, 1.0), 0.0)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_packed_layout_matches_numpy(ob):
    rng = np.random.default_rng(3)
    count, qpad = 37, 64
    k = _f16(rng, (count, H, D))
    v = _f16(rng, (H, D, count))
    q = rng.standard_normal((H, D)).astype(np.float32)
    mask = np.zeros((H, qpad, count), dtype=np.float32)
    mask[:, 0, rng.random(count) < 0.3] = -np.inf  # padded slots
    mask[5, 0, :] = -np.inf                         # a head with no live slot: zeros
    got = ob.attention_packed(_bits(k), _bits(v), mask, count, qpad, q)
    x = np.einsum("jhd,hd->hj", k.astype(np.float64), q.astype(np.float64)) * SCALE + mask[:, 0, :]
    want = np.einsum("hj,hdj->hd", _softmax(x), v.astype(np.float64))
    assert np.all(got[5] == 0.0)
    np.testing.assert_allclose(got, want, rtol=1e-11, atol=1e-13)


def test_compact_layout_matches_numpy(ob):
    rng = np.random.default_rng(4)
    count = 40
    lengths = rng.integers(0, count + 1, size=H).astype(np.uint32)
    lengths[0], lengths[1] = 0, count
    k = _f16(rng, (count, H, D))
    v = _f16(rng, (H, D, count))
    q = rng.standard_normal((H, D)).astype(np.float32)
    got = ob.attention_compact(_bits(k), _bits(v), count, lengths, q)
    for h in range(H):
        n = int(lengths[h])
        if n == 0:
            assert np.all(got[h] == 0.0)
            continue
        x = k[:n, h].astype(np.float64) @ q[h].astype(np.float64) * SCALE
        want = v[h, :, :n].astype(np.float64) @ _softmax(x)
        np.testing.assert_allclose(got[h], want, rtol=1e-11, atol=1e-13)


def test_dense_cache_matches_numpy(ob):
    rng = np.random.default_rng(5)
    n = 50
    kc = _f16(rng, (n, 8, D))
    vc = _f16(rng, (n, 8, D))
    q = rng.standard_normal((H, D)).astype(np.float32)
    got = ob.attention_dense(_bits(kc), _bits(vc), n, 1024, q)
    kh = np.arange(H) // 4
    x = np.einsum("thd,hd->ht", kc.astype(np.float64)[:, kh], q.astype(np.float64)) * SCALE
    want = np.einsum("ht,thd->hd", _softmax(x), vc.astype(np.float64)[:, kh])
    np.testing.assert_allclose(got, want, rtol=1e-11, atol=1e-13)


@pytest.mark.parametrize("threads", [1, 3])
def test_float_ports_stay_within_the_attention_tolerance(ob, threads):
    """The CPU baseline times float ports of the same graphs; they stay far
    inside the 2e-3 parity tolerance of the double-precision restatements."""
    rng = np.random.default_rng(6)
    count, qpad, n = 300, 64, 500
    k = _f16(rng, (count, H, D))
    v = _f16(rng, (H, D, count))
    q = rng.standard_normal((H, D)).astype(np.float32)
    mask = np.zeros((H, qpad, count), dtype=np.float32)
    mask[:, 0, count - 20:] = -np.inf
    exact = ob.attention_packed(_bits(k), _bits(v), mask, count, qpad, q)
    fast = ob.attention_packed_fast(_bits(k), _bits(v), mask, count, q, threads, qpad)
    assert np.max(np.abs(fast - exact)) / np.max(np.abs(exact)) < 1e-5
    kc = _f16(rng, (n, 8, D))
    vc = _f16(rng, (n, 8, D))
    exact = ob.attention_dense(_bits(kc), _bits(vc), n, 1024, q)
    fast = ob.attention_dense_fast(_bits(kc), _bits(vc), n, q, threads)
    assert np.max(np.abs(fast - exact)) / np.max(np.abs(exact)) < 1e-5


def test_rehearsal_matches_numpy(ob):
    """q = RoPE_position(W x): W bf16 [4096 out][4096 in], x bf16 [4096];
    NORM mode rotates adjacent channel pairs (2i, 2i+1) of each 128-wide head
    by position * theta^(-2i/128)."""
    rng = np.random.default_rng(7)

    def bf16(a):
        return (np.asarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)

    def widen(b):
        return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)

    x = bf16(rng.standard_normal(4096))
    w = bf16(rng.standard_normal((4096, 4096)) * 0.02)
    position, theta = 32768, 500000.0
    got = ob.rehearsal(x, w, position, theta)
    q = (widen(w) @ widen(x)).reshape(H, D // 2, 2)
    angle = position * theta ** (-2.0 * np.arange(D // 2) / D)
    c, s = np.cos(angle), np.sin(angle)
    want = np.stack([q[..., 0] * c - q[..., 1] * s, q[..., 0] * s + q[..., 1] * c], axis=-1).reshape(-1)
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-12)
