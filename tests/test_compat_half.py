"""The drop-in's binary16 conversions (hillserve::half_value / half_bits in
libhsb_compat, declared by compat/policy/host_policy.hpp) against the
reference's own (policy/host_policy.cpp:9-28, built into oracle/_ref), bit
for bit: every binary16 value widened, and narrowing at every value, every
midpoint between neighbours (the ties of round-to-nearest-even), one float
ulp either side of each midpoint, the overflow and underflow edges, signed
zeros, infinities and NaNs with payloads.  Host code only: CPU."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref" / "libhs_ref.so"


@pytest.fixture(scope="module")
def pair():
    from hillserve_b200 import build

    if not REF.exists():
        pytest.skip("reference library not built (reference sources absent at build time)")
    if not build.COMPAT_LIB.exists():
        build.build()
    compat, ref = C.CDLL(str(build.COMPAT_LIB)), C.CDLL(str(REF))
    ours_v, ours_b = compat._ZN9hillserve10half_valueEt, compat._ZN9hillserve9half_bitsEf
    ref_v, ref_b = ref.ref_half_value, ref.ref_half_bits
    for f in (ours_v, ref_v):
        f.argtypes, f.restype = [C.c_uint16], C.c_float
    for f in (ours_b, ref_b):
        f.argtypes, f.restype = [C.c_float], C.c_uint16
    return (ours_v, ours_b), (ref_v, ref_b)


def _f32_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float32).view(np.uint32)[0])


def test_widening_every_binary16(pair):
    (ours_v, _), (ref_v, _) = pair
    for h in range(65536):
        assert _f32_bits(ours_v(h)) == _f32_bits(ref_v(h)), hex(h)


def test_narrowing_at_values_ties_and_edges(pair):
    (_, ours_b), (_, ref_b) = pair
    finite = np.array([h for h in range(65536) if (h & 0x7C00) != 0x7C00], dtype=np.uint16)
    vals = np.sort(np.unique(finite.view(np.float16).astype(np.float64)))
    mids = (vals[:-1] + vals[1:]) / 2.0  # exact in float32: neighbouring halves differ in 11 bits
    f32 = np.concatenate([vals, mids]).astype(np.float32)
    up = np.nextafter(f32, np.float32(np.inf))
    down = np.nextafter(f32, np.float32(-np.inf))
    specials = np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65519.99, 65520.0, -65520.0, 1e9, -1e-9,
                         2.0 ** -24, 2.0 ** -25, 2.0 ** -25 * 1.0000001, 2.0 ** -26, 3e-8], dtype=np.float32)
    nans = np.array([0x7FC00000, 0xFFC00000, 0x7F800001, 0xFF812345, 0x7FBFFFFF], dtype=np.uint32).view(np.float32)
    rng = np.random.default_rng(11)
    rand = rng.integers(0, 2 ** 32, size=50000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for x in np.concatenate([f32, up, down, specials, nans, rand]):
        assert ours_b(float(x)) == ref_b(float(x)), hex(_f32_bits(float(x)))
