"""Seeded synthetic inputs for the parity tests (numpy, deterministic).

Config-1 style data: Q F16 [32,128] ~ N(0,1); K F16
[N,8,128] ~ N(0,1) with 2% of token rows (chosen uniformly, without
replacement) scaled x4 before rounding.  Normals come from a counter-based
splitmix64 hash and Box-Muller in float64, rounded to F16 by numpy (RNE), so
the same seed gives the same bits on every machine with this numpy.

Also reproduces the integer generator of the reference's scorer unit test
(the xorshift32 stream of tests/full_gqa_cpu_tests.cpp:19-27) so its vectors
can be rebuilt exactly, and draws kernel_check-style values
(kernels/full_gqa_pipeline/kernel_check.cpp:33-38).
"""
from __future__ import annotations

import hashlib

import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)) & _M
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _M
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _M
        return z ^ (z >> np.uint64(31))


def normals(seed: int, count: int, stream: int = 0) -> np.ndarray:
    """count N(0,1) float64 samples, one per counter."""
    i = np.arange(count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        base = splitmix64(np.uint64(seed) * np.uint64(0x100000001B3) + np.uint64(stream) * np.uint64(0x9E3779B9))
        u = splitmix64(i ^ base)
    u1 = ((u >> np.uint64(11)).astype(np.float64) + 0.5) / 9007199254740992.0
    u2 = ((splitmix64(u) >> np.uint64(11)).astype(np.float64) + 0.5) / 9007199254740992.0
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def heavy_rows(seed: int, n: int, fraction: float = 0.02) -> np.ndarray:
    """round(fraction*n) distinct token rows, uniformly chosen."""
    m = int(round(fraction * n))
    keys = splitmix64(np.arange(n, dtype=np.uint64) + np.uint64((seed * 0x5851F42D4C957F2D) % (1 << 64)))
    return np.sort(np.argsort(keys, kind="stable")[:m])


def config1(n: int = 4096, seed: int = 0, heavy_scale: float = 4.0):
    """(q [4096] uint16, k [n*1024] uint16, heavy row indices)."""
    q = f16_bits(normals(seed, 32 * 128, stream=1))
    kf = normals(seed, n * 1024, stream=2).reshape(n, 1024)
    heavy = heavy_rows(seed, n)
    kf[heavy] *= heavy_scale
    return q, f16_bits(kf).reshape(-1), heavy


def values(seed: int, n: int, stream: int = 3) -> np.ndarray:
    """V rows [n*1024] ~ N(0,1) F16 (unscaled)."""
    return f16_bits(normals(seed, n * 1024, stream=stream))


def interleave(k: np.ndarray, v: np.ndarray, n: int) -> np.ndarray:
    """Reference payload rows: K[8,128] then V[8,128] per token (2048 words)."""
    rows = np.empty((n, 2048), dtype=np.uint16)
    rows[:, :1024] = k.reshape(n, 1024)
    rows[:, 1024:] = v.reshape(n, 1024)
    return rows.reshape(-1)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


class XorShift32:
    """xorshift32 as in the reference tests (x^=x<<13; x^=x>>17; x^=x<<5)."""

    def __init__(self, state: int):
        self.s = state & 0xFFFFFFFF

    def __call__(self) -> int:
        s = self.s
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        self.s = s
        return s


_EDGE = [0, 0x8000, 1, 0x8001, 0x03FF, 0x83FF, 0x0400, 0x8400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF, 0x3555, 0xB555]


def cpu_test_half(rng: XorShift32) -> int:
    """finite_half() of tests/full_gqa_cpu_tests.cpp:21-27."""
    w = rng()
    if w % 5 == 0:
        return _EDGE[(w >> 8) % len(_EDGE)]
    return (w & 0x83FF) | (((w >> 10) % 31) << 10)


def pipeline_sample(rng: XorShift32) -> int:
    """A value drawn like sample() of kernels/full_gqa_pipeline/kernel_check.cpp
    :33-38: random sign, exponent field 0..16 (subnormals included), random
    mantissa -- finite and bounded so that sums do not overflow."""
    a = rng() & 0x8000
    b = (rng() % 17) << 10
    c = rng() & 1023
    return a | b | c


def cpu_test_case(rng: XorShift32, n: int, stride: int):
    """One (q, data) case of tests/full_gqa_cpu_tests.cpp:76-81: unused words
    of each row hold 0x7e00 (NaN), never read by the scorer."""
    q = np.array([cpu_test_half(rng) for _ in range(32 * 128)], dtype=np.uint16)
    data = np.full(n * stride, 0x7E00, dtype=np.uint16)
    for t in range(n):
        for c in range(1024):
            data[t * stride + c] = cpu_test_half(rng)
    return q, data


def h2o_probabilities(seed: int, first: int, queries: int, keys: int, heads: int = 32) -> np.ndarray:
    """Causal softmax-like rows, F32 [heads][queries][keys]: row (h, q) is
    w / sum(w) over keys 0..first+q (0 after), with integer weights w in
    1..1024 from splitmix64 (1 in 256 of them scaled by 1024: heavy hitters).
    Integer sums and one IEEE division per element make the values
    bit-reproducible on any platform."""
    n = heads * queries * keys
    x = splitmix64(np.arange(n, dtype=np.uint64) + np.uint64((seed * 0x9E3779B97F4A7C15) % (1 << 64)))
    w = ((x >> np.uint64(54)) + np.uint64(1)).astype(np.int64)
    w = np.where((x & np.uint64(0xff)) == 0, w << 10, w).reshape(heads, queries, keys)
    causal = np.arange(keys)[None, None, :] <= (first + np.arange(queries))[None, :, None]
    w = np.where(causal, w, 0)
    total = w.sum(axis=2, keepdims=True)
    return (w / total).astype(np.float32)


def h2o_layout(p: np.ndarray, ne0: int, ne1: int, nb0: int, nb1: int, nb2: int, fill=np.nan,
               total_bytes: int = 0) -> np.ndarray:
    """Places p [32][queries][keys] into a byte buffer with ggml strides (key
    nb0, query nb1, head nb2) over ne0 x ne1 x 32 elements; every byte not
    holding a valid probability is the F32 `fill` pattern (NaN by default),
    as in the reference's strided test."""
    heads, queries, keys = p.shape
    size = (ne0 - 1) * nb0 + (ne1 - 1) * nb1 + (heads - 1) * nb2 + 4
    size = max((size + 15) // 16 * 16, total_bytes)
    buf = np.full(size // 4, fill, dtype=np.float32).view(np.uint8)
    h, q, k = np.meshgrid(np.arange(heads), np.arange(queries), np.arange(keys), indexing="ij")
    offs = (k * nb0 + q * nb1 + h * nb2).reshape(-1)
    assert np.all(offs % 4 == 0)
    buf.view(np.float32)[offs // 4] = p.reshape(-1)
    return buf


def record_payload(seed: int, rows: int, record_bytes: int) -> np.ndarray:
    """Seeded payload bytes, uint8 [rows][record_bytes] (splitmix64 stream)."""
    n = (rows * record_bytes + 7) // 8
    x = splitmix64(np.arange(n, dtype=np.uint64) + np.uint64((seed * 0xD1B54A32D192ED03) % (1 << 64)))
    return x.view(np.uint8)[:rows * record_bytes].reshape(rows, record_bytes).copy()


def segment_image(request: int, layers: int, positions: int, record_bytes: int, payloads: list,
                  encode) -> np.ndarray:
    """The SegmentedKVStore v1 file holding payloads[l] at positions 0.. of
    layer l: a 4096-byte header, records at 4096 + (l*positions+p)*(B+32),
    zeros elsewhere, page-rounded extent.  `encode` makes the records."""
    stride = record_bytes + 32
    extent = (4096 + layers * positions * stride + 4095) // 4096 * 4096
    img = np.zeros(extent, dtype=np.uint8)
    words = np.zeros(512, dtype=np.uint64)
    words[:8] = [0x48534B5653454731, 1, request, layers, positions, record_bytes, stride, extent]
    img[:4096] = words.view(np.uint8)
    for l, rows in enumerate(payloads):
        if len(rows):
            recs = encode(rows, len(rows), record_bytes, request, l, 0)
            start = 4096 + l * positions * stride
            img[start:start + recs.nbytes] = recs
    return img
