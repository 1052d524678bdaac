"""Stage 2 parity on the GPU: the selector against the reference's known
answers, golden fixtures and the oracle (IDs, counts, k, ties bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from conftest import dev_u16, host_u16
from test_oracle_pin import _select_trial_input

pytestmark = pytest.mark.gpu
H = 32


def gsel(hsb, scores, heads, stride, valid, alpha, ratio, fp32=False, raw=False):
    s = hsb.select_gqa_scores(dev_u16(scores), heads, stride, valid, alpha, ratio, fp32, raw=raw)
    ids = s.ids.cpu().numpy().astype(np.uint64)
    return ids, np.array(s.counts, dtype=np.uint32), s.k, s.boundary_tied_heads


def same_as_oracle(hsb, ob, scores, heads, stride, valid, alpha, ratio, fp32=False):
    g = gsel(hsb, scores, heads, stride, valid, alpha, ratio, fp32)
    o = ob.select(scores, heads, stride, valid, alpha, ratio, fp32)
    assert g[2] == o[2], ("k", g[2], o[2])
    assert np.array_equal(g[1][:heads], o[1][:heads])
    assert np.array_equal(g[0], o[0])
    assert g[3] == o[3], ("ties", g[3], o[3])
    return g


def test_known_answers(cuda, ob):
    hb = ob.half_bits
    sc = np.array([hb(x) for x in (10, 9, 8, 7, 1, 1, 1, 1)], dtype=np.uint16)
    ids, counts, k, _ = same_as_oracle(cuda, ob, sc, 2, 4, 4, 2.0, 1.0)
    assert list(counts) == [3, 0] and k == 1 and ids[0, 0] == 0 and ids[1, 0] == 0
    pad = np.full(16, hb(1000), dtype=np.uint16)
    for h in range(2):
        for t in range(5):
            pad[h * 8 + t] = hb(float(t))
    ids, counts, k, _ = same_as_oracle(cuda, ob, pad, 2, 8, 5, 10, 0.4)
    assert k == 2 and list(ids[0]) == [4, 3]
    many = np.full(2049, hb(0), dtype=np.uint16)
    ids, counts, k, _ = same_as_oracle(cuda, ob, many, 1, 2049, 2049, 0, 1)
    assert counts[0] == 2049 and k == 2048
    ids, counts, k, _ = same_as_oracle(cuda, ob, many, 1, 2049, 2049, 0, 1, fp32=True)
    assert k == 2049
    long = np.full(131072, hb(-10), dtype=np.uint16)
    long[-1] = hb(1)
    ids, counts, k, _ = same_as_oracle(cuda, ob, long, 1, 131072, 131072, 0, 1)
    assert k == 1 and ids[0, 0] == 131071
    over = np.full(65520, hb(0), dtype=np.uint16)
    with pytest.raises(cuda.HsbError) as e:
        gsel(cuda, over, 1, 65520, 65520, 0, 1)
    assert e.value.status == 26 and "public F16 count overflow" in str(e.value)
    ids, counts, k, _ = same_as_oracle(cuda, ob, over, 1, 65520, 65520, 0, 0.2, fp32=True)
    assert counts[0] == 65520 and k == 13104 and ids[0, 0] == 0 and ids[0, -1] == 13103


def test_alpha_ramp_and_ties(cuda, ob):
    P = 128
    sc = np.array([ob.half_bits(100.0 - 2.0 * t) for _ in range(H) for t in range(P)], dtype=np.uint16)
    for alpha, kk, cc in zip((5, 10, 20, 50), (3, 6, 11, 25), (3, 6, 11, 26)):
        ids, counts, k, _ = same_as_oracle(cuda, ob, sc, H, P, P, alpha, 0.2)
        assert k == kk and np.all(counts == cc)
    for alpha in (5.0, 10.0, 20.0, 50.0):
        sc = np.full(H * P, ob.half_bits(-1000.0), dtype=np.uint16)
        tb = ob.half_bits(100.0 - alpha)
        for h in range(H):
            sc[h * P:h * P + 4] = [ob.half_bits(100.0), tb, tb, tb - 1]
        ids, counts, k, _ = same_as_oracle(cuda, ob, sc, H, P, P, alpha, 0.2)
        assert k == 3 and list(ids[0]) == [0, 1, 2]
        sc[0] = ob.half_bits(120.0)
        same_as_oracle(cuda, ob, sc, H, P, P, alpha, 0.2)


def test_2049_rounding_n16384(cuda, ob):
    N = 16384
    sc = np.full(H * N, ob.half_bits(-1000.0), dtype=np.uint16)
    for h in range(H):
        sc[h * N:h * N + 2049] = ob.half_bits(0.0)
    for alpha in (5.0, 50.0):
        ids, counts, k, _ = same_as_oracle(cuda, ob, sc, H, N, N, alpha, 0.2)
        assert k == 2048 and counts[0] == 2049 and ids[0, -1] == 2047


def test_random_trials_golden(cuda, golden):
    g = golden("select_trials.npz")
    rng = inputs.XorShift32(1741)
    for trial in range(24):
        x = _select_trial_input(rng, 32, 257, 288)
        i = g["names"].tolist().index(f"t{trial}")
        ids, counts, k, tied = gsel(cuda, x, 32, 288, 257, 10.0, 0.2)
        assert k == g["k"][i] and tied == g["tied"][i]
        assert inputs.digest(ids) == g["ids_digest"][i]
        assert inputs.digest(counts) == g["counts_digest"][i]


@pytest.mark.parametrize("n", [64, 1024, 4096, 16384])
def test_config1_alpha_sweep_golden(cuda, golden, n):
    """Scored on the GPU, normalised in the selector (raw input), selected:
    against the reference's k, counts and ordered IDs."""
    import torch

    g = golden(f"config1_n{n}.npz")
    q, k, _ = inputs.config1(n, seed=0)
    raw = cuda.score_full_gqa(dev_u16(q), [(dev_u16(k), n, 1024)])
    scaled = cuda.scale_scores(raw)
    torch.cuda.synchronize()
    assert inputs.digest(host_u16(scaled)) == g["scaled_digest"]
    for a in g["alphas"]:
        tag = f"a{float(a):g}".replace(".", "p")
        for use_raw, src in ((True, raw), (False, scaled)):
            s = cuda.select_gqa_scores(src, H, n, n, float(a), 0.2, raw=use_raw)
            assert s.k == g[f"{tag}_k"] and s.boundary_tied_heads == g[f"{tag}_tied"]
            assert np.array_equal(np.array(s.counts, dtype=np.uint32), g[f"{tag}_counts"])
            ids = s.ids.cpu().numpy().astype(np.uint32)
            assert inputs.digest(ids) == g[f"{tag}_ids_digest"]


@pytest.mark.parametrize("n,alpha", [(32768, 0.1), (32768, 5.0), (32768, 10.0), (32768, 50.0), (20000, 3.0),
                                     (70000, 2.0)])
def test_large_vs_oracle(cuda, ob, n, alpha):
    rng = np.random.default_rng(n)
    vals = (rng.standard_normal(H * n) * (1 + 3 * (rng.random(H * n) < 0.02))).astype(np.float16)
    sc = vals.view(np.uint16).copy()
    same_as_oracle(cuda, ob, sc, H, n, n, alpha, 0.2)


def test_coarse_values_many_ties(cuda, ob):
    """Few distinct values: K* ties dominate, boundary ties and +-0 appear."""
    rng = np.random.default_rng(3)
    n = 5000
    vals = rng.integers(-4, 5, size=H * n).astype(np.float16)
    sc = vals.view(np.uint16).copy()
    sc[::7] ^= (0x8000 * (sc[::7] == 0)).astype(np.uint16)  # some -0
    for alpha in (0.0, 1.0, 3.0, 8.0):
        for ratio in (0.2, 0.5, 1.0):
            same_as_oracle(cuda, ob, sc, H, n, n, alpha, ratio)


@pytest.mark.parametrize("n,seed", [(32768, 1), (32768, 2), (20000, 3), (4100, 4)])
def test_few_candidates_with_equal_top_keys(cuda, ob, n, seed):
    """Equal top keys spread over the four chunks of a head, few enough that
    the selector's direct path places them in arrival order (at most 256
    candidates): the selection must still list equal keys by ascending ID,
    and heads holding more equal keys than k count as boundary ties."""
    rng = np.random.default_rng(seed)
    sc = rng.standard_normal((H, n)).astype(np.float16)
    for h in range(H):
        planted = rng.choice(n, size=8 + h % 5, replace=False)  # 8..12 copies of the maximum
        sc[h, planted] = np.float16(6.0)
        second = rng.choice(np.setdiff1d(np.arange(n), planted), size=3, replace=False)
        sc[h, second] = np.float16(5.75)  # a second tier just below
    bits = sc.view(np.uint16).reshape(-1).copy()
    for alpha in (0.2, 0.3, 1.0):
        g = same_as_oracle(cuda, ob, bits, H, n, n, alpha, 0.2)
        assert g[2] > 0


def test_errors_in_reference_order(cuda, ob):
    hb = ob.half_bits
    n = 64
    base = np.full(H * n, hb(0.5), dtype=np.uint16)
    bad0 = base.copy()
    bad0[5] = 0x7C00
    with pytest.raises(cuda.HsbError) as e:
        gsel(cuda, bad0, H, n, n, 1.0, 0.2)
    assert e.value.status == 22 and str(e.value) == "nonfinite head0 score"
    bad3 = base.copy()
    bad3[3 * n + 9] = 0x7E00
    bad3[7 * n + 1] = 0x7C00
    with pytest.raises(cuda.HsbError) as e:
        gsel(cuda, bad3, H, n, n, 1.0, 0.2)
    assert e.value.status == 24 and str(e.value) == "nonfinite GQA score"
    low = np.full(H * n, hb(-65504.0), dtype=np.uint16)
    with pytest.raises(cuda.HsbError) as e:
        gsel(cuda, low, H, n, n, 100.0, 0.2)
    assert e.value.status == 23
    # padding beyond valid is never read: infinities there are fine
    padded = base.copy().reshape(H, n)
    padded[:, 40:] = 0x7C00
    same_as_oracle(cuda, ob, padded.reshape(-1), H, n, 40, 1.0, 0.2)


def _keys_select(hsb, raw_dev, heads, n, alpha, ratio=0.2):
    """hsb_select_keys on keys derived on the GPU from raw scores."""
    import torch

    lib = hsb._capi.lib()
    s = torch.cuda.current_stream().cuda_stream
    keys = torch.empty_like(raw_dev)
    # scale then key on the GPU: the scorer path is exercised separately below
    kcap = max(1, hsb.select_kmax(n, ratio))
    ids = torch.empty((heads, kcap), dtype=torch.int32, device="cuda")
    counts = torch.zeros(heads, dtype=torch.int32, device="cuda")
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = hsb._workspace(lib.hsb_select_workspace_bytes(heads, n, n, kcap), "cuda")
    return lib, s, keys, ids, counts, res, ws, kcap


@pytest.mark.parametrize("n,alpha", [(4096, 0.1), (4096, 10.0), (32768, 5.0), (32768, 50.0), (5000, 3.0)])
def test_score_with_keys_then_select_keys(cuda, ob, n, alpha):
    """The fused pipeline path: the scorer emits order keys of normalised
    scores, the selector consumes them -- same IDs/counts/k/ties as the
    reference chain score -> scale -> select."""
    import ctypes as C

    import torch

    q, k, _ = inputs.config1(n, seed=9)
    lib, s, keys, ids, counts, res, ws, kcap = _keys_select(cuda, torch.empty((32, n), dtype=torch.int16,
                                                                                device="cuda"), 32, n, alpha)
    raw = torch.empty((32, n), dtype=torch.int16, device="cuda")
    assert lib.hsb_score_with_keys(dev_u16(q).data_ptr(), dev_u16(k).data_ptr(), n, 1024, raw.data_ptr(),
                                   keys.data_ptr(), s) == 0
    assert lib.hsb_select_keys(keys.data_ptr(), raw.data_ptr(), 32, n, n, C.c_float(alpha), C.c_float(0.2), 0,
                               ids.data_ptr(), kcap, counts.data_ptr(), res.data_ptr(), ws.data_ptr(), ws.numel(),
                               s) == 0
    torch.cuda.synchronize()
    raw_h = ob.score(q, k, n, 1024)
    assert np.array_equal(host_u16(raw), raw_h)
    scaled = ob.scale(raw_h)
    want_keys = np.array([ob.oracle().orc_order_key(int(b)) for b in scaled.reshape(-1)[:4096]], dtype=np.uint16)
    assert np.array_equal(host_u16(keys).reshape(-1)[:4096], want_keys)
    wids, wcounts, wk, wtied = ob.select(scaled, 32, n, n, alpha, 0.2)
    r = res.cpu().numpy()
    assert r[0] == wk and r[1] == wtied and r[2] == 0
    assert np.array_equal(counts.cpu().numpy().astype(np.uint32), wcounts)
    assert np.array_equal(ids[:, :wk].cpu().numpy().astype(np.uint64), wids)


def test_select_keys_signed_zero_ties(cuda, ob):
    """Keys lose the sign of zero; the boundary-tie rule reads it back from the
    raw scores (gqa_policy.cpp:66 compares F16 bits, so +0 / -0 differ)."""
    import ctypes as C

    import torch

    n = 512
    rng = np.random.default_rng(8)
    raw = np.where(rng.random(32 * n) < 0.5, 0x0000, 0x8000).astype(np.uint16)  # only +0 / -0
    raw[rng.random(32 * n) < 0.01] = ob.half_bits(8.0)
    scaled = ob.scale(raw)
    keys = np.array([ob.oracle().orc_order_key(int(b)) for b in scaled], dtype=np.uint16)
    for alpha in (0.0, 0.5, 20.0):
        lib, s, _, ids, counts, res, ws, kcap = _keys_select(cuda, dev_u16(raw), 32, n, alpha)
        assert lib.hsb_select_keys(dev_u16(keys).data_ptr(), dev_u16(raw).data_ptr(), 32, n, n, C.c_float(alpha),
                                   C.c_float(0.2), 0, ids.data_ptr(), kcap, counts.data_ptr(), res.data_ptr(),
                                   ws.data_ptr(), ws.numel(), s) == 0
        torch.cuda.synchronize()
        wids, wcounts, wk, wtied = ob.select(scaled, 32, n, n, alpha, 0.2)
        r = res.cpu().numpy()
        assert r[0] == wk and r[1] == wtied
        assert np.array_equal(ids[:, :wk].cpu().numpy().astype(np.uint64), wids)
