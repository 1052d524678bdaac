"""Pins the C oracle to the reference: the reference tests' own known-answer
vectors, exhaustive binary16 checks, and golden fixtures produced by running
the reference's code (tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

import inputs

H, D = 32, 128


# ------------------------------------------------------------------ half
def test_half_roundtrip_exhaustive(ob):
    # tests/policy_tests.cpp:8: every non-NaN binary16 survives a round trip.
    bits = np.arange(65536, dtype=np.uint16)
    lib = ob.oracle()
    for b in bits:
        if (b & 0x7C00) == 0x7C00 and (b & 0x3FF):
            continue
        assert lib.orc_half_bits(lib.orc_half_value(int(b))) == b


def test_half_rne_known_answers(ob):
    # tests/policy_tests.cpp:9-10
    assert ob.half_bits(1.00048828125) == ob.half_bits(1.0)
    assert ob.half_bits(1.00146484375) == ob.half_bits(1.001953125)
    assert ob.half_bits(65520.0) == 0x7C00 and ob.half_bits(65519.0) == 0x7BFF
    assert ob.half_bits(float("nan")) == 0x7E00


def test_half_matches_numpy_rne(ob):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(20000) * 10 ** rng.uniform(-9, 5, 20000),
                        rng.uniform(-7e4, 7e4, 2000)]).astype(np.float32)
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([ob.half_bits(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(got, want)


def test_order_key_exhaustive(ob):
    # tests/gqa_policy_tests.cpp:42-48: key order == FP32 comparator order.
    finite = [b for b in range(65536) if (b & 0x7C00) != 0x7C00]
    vals = np.array([ob.half_value(b) for b in finite])
    order = np.argsort(vals, kind="stable")
    keys = np.array([ob.oracle().orc_order_key(finite[i]) for i in order])
    v = vals[order]
    assert np.all((keys[1:] > keys[:-1]) == (v[1:] > v[:-1]))
    assert np.all((keys[1:] == keys[:-1]) == (v[1:] == v[:-1]))


# ------------------------------------------------------------------ scorer
def test_scorer_reference_test_vectors(ob, golden):
    """The xorshift vectors of tests/full_gqa_cpu_tests.cpp:76-86, against the
    digests of the reference's own scores."""
    g = golden("scorer_vectors.npz")
    want = dict(zip(g["names"].tolist(), zip(g["input_digest"].tolist(), g["score_digest"].tolist())))
    rng = inputs.XorShift32(0x7F123451)
    checked = 0
    for n in (1, 2, 7, 8, 9, 17, 65, 129):
        for stride in (1024, 2048):
            q, data = inputs.cpu_test_case(rng, n, stride)
            din, dsc = want[f"n{n}_s{stride}"]
            assert inputs.digest(q, data) == din
            assert inputs.digest(ob.score(q, data, n, stride)) == dsc
            checked += 1
            if n >= 9:
                views = [(data, 7 * stride, 2, stride), (data, 0, 3, stride), (data, stride, 1, stride)]
                assert inputs.digest(ob.score_views(q, views)) == want[f"n{n}_s{stride}_views"][1]
    assert checked == 16


def _pipeline_markers(n: int):
    """kernel_check.cpp:79-92 marker construction (positive and negative
    subnormal markers, ordered cancellation on head 31)."""
    rng = inputs.XorShift32(0x62C83E17)
    q = np.array([inputs.pipeline_sample(rng) for _ in range(4096)], dtype=np.uint16)
    k = np.array([inputs.pipeline_sample(rng) for _ in range(n * 1024)], dtype=np.uint16)
    q[:128] = 0
    q[0] = 0x3C00
    q[28 * 128:29 * 128] = 0
    q[28 * 128 + 3] = 0x3C00
    q[31 * 128:] = 0
    q[31 * 128] = 0x6C00
    q[31 * 128 + 1] = 0x3C00
    q[31 * 128 + 2] = 0xEC00
    for t in range(n):
        k[t * 1024] = t + 1
        last = (t * 8 + 7) * 128
        k[last] = 0x6C00
        k[last + 1] = 0x3C00
        k[last + 2] = 0x6C00
        k[last + 3] = 0x8000 | (t + 1)
    return q, k


def test_scorer_kernel_check_markers(ob):
    # kernel_check.cpp:93-98: exact known answers.
    n = 192
    q, k = _pipeline_markers(n)
    s = ob.score(q, k, n, 1024)
    t = np.arange(n)
    assert np.array_equal(s[0], (t + 1).astype(np.uint16))
    assert np.array_equal(s[28], (0x8000 | (t + 1)).astype(np.uint16))
    assert np.all(s[31] == 0)  # 4096*4096 + 1 - 4096*4096 == 0 in order


def test_scorer_edge_fills(ob):
    # full_gqa_cpu_tests.cpp:87-97: subnormal minimum, cancellation, overflow, -0.
    n = 9
    q = np.ones(4096, dtype=np.uint16)
    data = np.ones(9 * 1024, dtype=np.uint16)
    s = ob.score(q, data, n, 1024)
    assert np.all(s == ob.half_bits(128 * 2.0 ** -48))  # underflows to +0 in F16
    q = np.where(np.arange(4096) % 2, 0xFBFF, 0x7BFF).astype(np.uint16)
    data[:] = 0x7BFF
    assert np.all(ob.score(q, data, n, 1024) == 0)
    q[:] = 0x7BFF
    assert np.all(ob.score(q, data, n, 1024) == 0x7C00)
    q[:] = 0x8000
    assert np.all(ob.score(q, data, n, 1024) == 0)  # +0 + (-0 products) stays +0


def test_fma_equals_mul_add_on_f16_products():
    """The sm_100a scorer issues one FMA per (head, channel).  That equals the
    reference's rounded multiply then add because a product of two binary16
    values is exact in binary32; checked here on random and extreme values."""
    rng = np.random.default_rng(11)
    bits = rng.integers(0, 65536, size=200000, dtype=np.uint32).astype(np.uint16)
    bits = bits[(bits & 0x7C00) != 0x7C00]
    a = bits[: len(bits) // 2].view(np.float16).astype(np.float64)
    b = bits[len(bits) // 2: 2 * (len(bits) // 2)].view(np.float16).astype(np.float64)
    prod64 = a * b
    assert np.array_equal(prod64.astype(np.float32).astype(np.float64), prod64)  # exact in binary32


# ------------------------------------------------------------------ selector
def test_selector_known_answers(ob):
    hb = ob.half_bits
    # gqa_policy_tests.cpp:25-26: head0 broadcast + inclusive; counts {3,0}, k=1
    sc = np.array([hb(x) for x in (10, 9, 8, 7, 1, 1, 1, 1)], dtype=np.uint16)
    ids, counts, k, tied = ob.select(sc, 2, 4, 4, 2.0, 1.0)
    assert list(counts[:2]) == [3, 0] and k == 1 and ids[0, 0] == 0 and ids[1, 0] == 0
    # :28-29 padding is not a candidate
    pad = np.full(16, hb(1000), dtype=np.uint16)
    for h in range(2):
        for t in range(5):
            pad[h * 8 + t] = hb(float(t))
    ids, counts, k, tied = ob.select(pad, 2, 8, 5, 10, 0.4)
    assert k == 2 and list(ids[0]) == [4, 3]
    # :31 F16 count rounding 2049 -> 2048
    many = np.full(2049, hb(0), dtype=np.uint16)
    ids, counts, k, tied = ob.select(many, 1, 2049, 2049, 0, 1)
    assert counts[0] == 2049 and k == 2048
    # :33 long IDs
    long = np.full(131072, hb(-10), dtype=np.uint16)
    long[-1] = hb(1)
    ids, counts, k, tied = ob.select(long, 1, 131072, 131072, 0, 1)
    assert k == 1 and ids[0, 0] == 131071
    # :34 F16 count overflow rejects; :37-40 FP32 extension
    over = np.full(65520, hb(0), dtype=np.uint16)
    with pytest.raises(ob.OracleError) as e:
        ob.select(over, 1, 65520, 65520, 0, 1)
    assert e.value.code == 26
    ids, counts, k, tied = ob.select(over, 1, 65520, 65520, 0, 0.2, fp32_counts=True)
    assert counts[0] == 65520 and k == 13104 and ids[0, 0] == 0 and ids[0, -1] == 13103
    ids, counts, k, tied = ob.select(many, 1, 2049, 2049, 0, 1, fp32_counts=True)
    assert k == 2049


def test_selector_alpha_ramp(ob):
    # tests/quality_alpha_tests.cpp:35-47: alpha -> k {3,6,11,25}, counts {3,6,11,26}
    P = 128
    sc = np.array([ob.half_bits(100.0 - 2.0 * t) for _ in range(H) for t in range(P)], dtype=np.uint16)
    for alpha, kk, cc in zip((5, 10, 20, 50), (3, 6, 11, 25), (3, 6, 11, 26)):
        ids, counts, k, tied = ob.select(sc, H, P, P, alpha, 0.2)
        assert k == kk and np.all(counts == cc)
        assert np.all(ids == np.arange(k))


def test_selector_threshold_ties_and_head0(ob):
    # quality_alpha_tests.cpp:49-66
    P = 128
    for alpha in (5.0, 10.0, 20.0, 50.0):
        sc = np.full(H * P, ob.half_bits(-1000.0), dtype=np.uint16)
        tb = ob.half_bits(100.0 - alpha)
        for h in range(H):
            sc[h * P] = ob.half_bits(100.0)
            sc[h * P + 1] = tb
            sc[h * P + 2] = tb
            sc[h * P + 3] = tb - 1
        ids, counts, k, tied = ob.select(sc, H, P, P, alpha, 0.2)
        assert k == 3 and counts[0] == 3 and list(ids[0]) == [0, 1, 2]
        sc[0] = ob.half_bits(120.0)
        ids, counts, k, tied = ob.select(sc, H, P, P, alpha, 0.2)
        new_thr = ob.half_value(ob.half_bits(120.0 - alpha))
        assert counts[1] == int(100.0 >= new_thr)


def test_selector_2049_rounding_n16384(ob):
    # quality_alpha_tests.cpp:70-77
    N = 16384
    sc = np.full(H * N, ob.half_bits(-1000.0), dtype=np.uint16)
    for h in range(H):
        sc[h * N: h * N + 2049] = ob.half_bits(0.0)
    for alpha in (5.0, 10.0, 20.0, 50.0):
        ids, counts, k, tied = ob.select(sc, H, N, N, alpha, 0.2)
        assert k == 2048 and counts[0] == 2049 and ids[0, -1] == 2047


def test_selector_random_trials_golden(ob, golden):
    g = golden("select_trials.npz")
    rng = inputs.XorShift32(1741)
    for trial in range(24):
        heads, n, stride = 32, 257, 288
        x = _select_trial_input(rng, heads, n, stride)
        i = g["names"].tolist().index(f"t{trial}")
        assert inputs.digest(x) == g["input_digest"][i]
        ids, counts, k, tied = ob.select(x, heads, stride, n, 10.0, 0.2)
        assert k == g["k"][i] and tied == g["tied"][i]
        assert inputs.digest(ids.astype(np.uint64)) == g["ids_digest"][i]
        assert inputs.digest(counts) == g["counts_digest"][i]
        # and against a full sort (gqa_policy_tests.cpp:55-57)
        for h in range(heads):
            vals = np.array([ob.half_value(int(b)) for b in x[h * stride:h * stride + n]])
            order = sorted(range(n), key=lambda t: (-vals[t], t))[:k]
            assert list(ids[h]) == order


def _select_trial_input(rng, heads, n, stride):
    x = np.full(heads * stride, inputs.f16_bits(np.float32(1000.0)), dtype=np.uint16)
    for h in range(heads):
        for t in range(n):
            if t % 17 == 0:
                x[h * stride + t] = 0 if t % 2 else 0x8000
            else:
                x[h * stride + t] = inputs.f16_bits(np.float32((int(rng() % 97) - 48) / 2))
    return x


@pytest.mark.parametrize("n", [64, 1024, 4096])
def test_config1_golden(ob, golden, n):
    """Config 1 (and config-3 lengths): raw scores, scaling and the alpha sweep
    against the reference's outputs."""
    g = golden(f"config1_n{n}.npz")
    q, k, _ = inputs.config1(n, seed=0)
    assert inputs.digest(q, k) == g["input_digest"]
    raw = ob.score(q, k, n, 1024)
    assert inputs.digest(raw) == g["raw_digest"]
    scaled = ob.scale(raw)
    assert inputs.digest(scaled) == g["scaled_digest"]
    for a in g["alphas"]:
        tag = f"a{float(a):g}".replace(".", "p")
        ids, counts, kk, tied = ob.select(scaled, H, n, n, float(a), 0.2)
        assert kk == g[f"{tag}_k"] and tied == g[f"{tag}_tied"]
        assert np.array_equal(counts, g[f"{tag}_counts"])
        assert inputs.digest(ids.astype(np.uint32)) == g[f"{tag}_ids_digest"]


# ------------------------------------------------------------------ pack
def test_pack_known_answers(ob):
    # tests/gqa_pack_tests.cpp:7-14
    ids = np.tile(np.array([8, 12], dtype=np.uint64), (32, 1))
    ids[4] = [12, 8]
    physical = np.array([8, 12], dtype=np.uint64)
    raw = np.zeros(4096, dtype=np.uint16)
    for t in range(2):
        for h in range(8):
            for d in range(128):
                raw[t * 2048 + h * 128 + d] = 1000 * t + 100 * h + d
                raw[t * 2048 + 1024 + h * 128 + d] = 5000 + 1000 * t + 100 * h + d
    payload = raw.view(np.uint8)
    k, v, mask = ob.pack(ids, [2] * 32, [10, 12], physical, payload, 32)
    assert k[0] == 0 and k[4096] == 1000 and k[4 * 128] == 1100 and k[4096 + 4 * 128] == 100
    assert v[(4 * 128) * 32] == 6100 and v[(4 * 128) * 32 + 1] == 5100
    assert k[2 * 4096 + 127] == 0 and v[127 * 32 + 2] == 0
    assert mask[0] == 0 and np.isinf(mask[1]) and mask[32 + 1] == 0
    assert np.isinf(mask[(4 * 64) * 32]) and mask[(4 * 64) * 32 + 1] == 0 and np.isinf(mask[2 * 32])
    bad = np.vstack([np.array([[13, 0]], dtype=np.uint64), ids[1:]])  # ids[0] = {13}
    with pytest.raises(ob.OracleError) as e:
        ob.pack(bad, [1] + [2] * 31, [12], physical, payload, 32)
    assert e.value.code == 43


def test_pack_and_union_golden(ob, golden):
    from golden.make_golden import pack_case

    g = golden("pack_trials.npz")
    for i, name in enumerate(g["names"].tolist()):
        trial = int(name[1:])
        ids, sizes, positions, rows, payload, slots = pack_case(trial)
        assert inputs.digest(ids, sizes, positions, rows, payload) == g["input_digest"][i]
        k, v, mask = ob.pack(ids, sizes, positions, rows, payload, slots)
        assert inputs.digest(k) == g["k_digest"][i]
        assert inputs.digest(v) == g["v_digest"][i]
        assert inputs.digest(mask) == g["mask_digest"][i]
        assert inputs.digest(ob.union(ids, sizes, len(rows))) == g["union_digest"][i]


def test_union_rejects_duplicates(ob):
    ids = np.zeros((32, 3), dtype=np.uint64)
    ids[:, 0] = 1
    ids[:, 1] = 2
    sizes = [2] * 32
    assert list(ob.union(ids, sizes, 5)) == [1, 2]
    ids[31, 2] = 1
    sizes[31] = 3
    with pytest.raises(ob.OracleError):
        ob.union(ids, sizes, 5)
    with pytest.raises(ob.OracleError):
        ob.union(ids, [2] * 32, 2)  # id 2 is not visible


# ------------------------------------------------------------------ cover
def _cover_key(layer, pos, head, d):
    """key() of tests/full_gqa_prefetch_tests.cpp:27-32."""
    if d:
        return 0.0
    value = (pos % 16) * 0.25 + (layer % 8) * 0.125 + head * 0.03125
    if pos >= 128:
        value = (512.0 if layer % 2 == 0 else -512.0) + float(pos - 128)
    return value


@pytest.mark.parametrize("layer", [0, 1, 2, 3])
@pytest.mark.parametrize("position", [128, 129, 140])
def test_prefetch_cover_bounds_and_cover(ob, layer, position):
    """Cover property (full_gqa_prefetch_tests.cpp:47-55, 195-205): every final
    selected ID of the history is in the prefetched cover, and the per-head
    bound is the F16 threshold-count upper bound."""
    capacity = 192
    hb = ob.half_bits
    # raw scores with query q[h*128]=1: score = key(layer,t,h/4,0)
    raw = np.zeros(32 * capacity, dtype=np.uint16)
    for h in range(32):
        for t in range(position + 1):
            raw[h * capacity + t] = hb(_cover_key(layer, t, h // 4, 0))
    per_head, physical = ob.prefetch_cover(raw, capacity, position, 5.0)
    cap = int(np.floor((position + 1) * float(np.float32(0.2))))
    expected = min(cap, position - 128 + 1) if (layer % 2 == 0 and position > 128) else cap
    assert per_head.shape[1] == expected
    assert np.all(per_head < position)
    scaled = ob.scale(raw)
    ids, counts, k, tied = ob.select(scaled, 32, capacity, position + 1, 5.0, 0.2)
    final = set(int(i) for i in ids.reshape(-1) if i < position)
    assert final <= set(int(i) for i in physical)
