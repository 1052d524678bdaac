"""The CPU restatement of the benchmark input generator (oracle/
orc_synth_*), pinned against the same definition evaluated with numpy's
libm (float64 log/cos/sin): Box-Muller normals, heavy rows and NORM-mode
RoPE.  The restatement's own series must agree with libm to well below one
F16 rounding, so its F16 (and BF16) bits equal libm's on every sample that is
not within a hair of a rounding boundary."""
from __future__ import annotations

import numpy as np
import pytest

from inputs import splitmix64

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def _uniforms(seed: int, idx: np.ndarray):
    with np.errstate(over="ignore"):
        a = splitmix64(np.uint64(seed) ^ splitmix64(idx.astype(np.uint64)))
        b = splitmix64(a)
    u1 = ((a >> np.uint64(12)).astype(np.float64) + 0.5) * 2.0 ** -52
    u2 = ((b >> np.uint64(12)).astype(np.float64) + 0.5) * 2.0 ** -52
    return u1, u2


def _libm_normal(seed: int, idx: np.ndarray) -> np.ndarray:
    u1, u2 = _uniforms(seed, idx)
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float32).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("seed,stddev", [(0, 1.0), (12345, 1.0), (7, 0.02)])
def test_normals_match_libm(ob, seed, stddev):
    n = 1 << 20
    want = _f16(_libm_normal(seed, np.arange(n)) * float(np.float32(stddev)))  # the C ABI takes a float
    got = ob.synth_normal(n, seed, stddev)
    assert np.count_nonzero(got != want) <= n // 100000  # boundary cases only
    v = got.view(np.float16).astype(np.float64) / stddev
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01


def test_bf16_rounding(ob):
    n = 1 << 18
    z = (_libm_normal(99, np.arange(n)) * float(np.float32(0.02))).astype(np.float32).view(np.uint32)
    want = ((z + np.uint32(0x7FFF) + ((z >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    got = ob.synth_normal(n, 99, 0.02, bf16=True)
    assert np.count_nonzero(got != want) <= 2


def test_keys_heavy_rows_and_rope(ob):
    tokens, seed = 4096, 3
    plain = ob.synth_keys(tokens, seed, rope=False).reshape(tokens, 1024)
    with np.errstate(over="ignore"):
        h = splitmix64((np.uint64(seed) * np.uint64(0x2545F4914F6CDD1D) + np.arange(tokens, dtype=np.uint64)) & _M)
    heavy = h < np.uint64(int(float(np.float32(0.02)) * 2.0 ** 64))
    base = _libm_normal(seed, np.arange(tokens * 1024)).reshape(tokens, 1024)
    want = _f16(np.where(heavy[:, None], base * 4.0, base))
    assert np.count_nonzero(plain != want) <= 2
    assert 0.01 < heavy.mean() < 0.03
    # NORM-mode rotation of pair (2i, 2i+1) of every KV head by t * theta^(-i/64)
    rot = ob.synth_keys(tokens, seed, rope=True).reshape(tokens, 1024)
    x = np.where(heavy[:, None], base * 4.0, base)
    i = (np.arange(512) % 64).astype(np.float64)
    ang = np.arange(tokens)[:, None] * 500000.0 ** (-i / 64.0)[None, :]
    a, b = x[:, 0::2], x[:, 1::2]
    ra = a * np.cos(ang) - b * np.sin(ang)
    rb = a * np.sin(ang) + b * np.cos(ang)
    want_r = np.empty_like(x)
    want_r[:, 0::2], want_r[:, 1::2] = ra, rb
    diff = rot.view(np.float16).astype(np.float64) - _f16(want_r).view(np.float16).astype(np.float64)
    assert np.count_nonzero(diff) <= tokens * 1024 // 5000
    # where they differ it is one F16 step of the value, never more
    ulp = np.spacing(np.abs(want_r).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(diff) <= ulp * 1.0001)


def test_threads_do_not_change_bits(ob):
    a = ob.synth_keys(1000, 17, threads=1)
    b = ob.synth_keys(1000, 17, threads=7)
    assert np.array_equal(a, b)
