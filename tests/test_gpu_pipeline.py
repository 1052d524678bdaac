"""End-to-end on the GPU: the rehearsal query producer, the prefetch cover, and
the fused selected-KV layer step (score -> select -> gather -> attention)
against the oracle chain (scores, IDs and gathered K/V bit-exact, attention
within 2e-3)."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from conftest import dev_u16, host_u16

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _t(a, dtype):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to("cuda")


def test_rehearsal_query(cuda, ob):
    """Config 4's producer: x bf16 ~ N(0,1), W bf16 ~ N(0,0.02), RoPE at N.
    Parity is unpinned (ggml); the oracle is FP64.  The F16 output is the RNE
    cast of the F32 output, bit-exactly."""
    import torch

    x = torch.randn(4096, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(4096, 4096, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    for position in (0, 1, 4097, 32768):
        q32, q16 = cuda.rehearsal_query(x.cuda(), w.cuda(), position, 500000.0)
        torch.cuda.synchronize()
        want = ob.rehearsal(x.view(torch.int16).numpy().view(np.uint16), w.view(torch.int16).numpy().view(np.uint16),
                            position, 500000.0)
        got = q32.cpu().numpy().reshape(-1).astype(np.float64)
        assert np.max(np.abs(got - want)) <= 1e-4 * np.max(np.abs(want))
        assert np.array_equal(host_u16(q16).reshape(-1), q32.cpu().numpy().reshape(-1).astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("position,layer", [(128, 0), (129, 2), (140, 1), (1000, 3)])
def test_prefetch_cover(cuda, ob, position, layer):
    import torch
    from test_oracle_pin import _cover_key

    capacity = max(192, position + 8)
    raw = np.zeros(32 * capacity, dtype=np.uint16)
    for h in range(32):
        for t in range(position + 1):
            raw[h * capacity + t] = ob.half_bits(_cover_key(layer, t, h // 4, 0) + (t % 7) * 0.01 * h)
    per_head, physical = cuda.prefetch_cover(dev_u16(raw), capacity, position, 5.0)
    torch.cuda.synchronize()
    wper, wphys = ob.prefetch_cover(raw, capacity, position, 5.0)
    assert np.array_equal(per_head.cpu().numpy().astype(np.uint64), wper)
    assert np.array_equal(physical.cpu().numpy().astype(np.uint64), wphys)


def oracle_layer(ob, q16, q32, k, v, n, alpha):
    raw = ob.score(q16, k, n, 1024)
    scaled = ob.scale(raw)
    ids, counts, kk, tied = ob.select(scaled, 32, n, n, alpha, 0.2)
    return raw, ids, counts, kk


@pytest.mark.parametrize("n,alpha", [(4096, 10.0), (4096, 5.0), (4096, 0.1), (16384, 10.0), (32768, 10.0),
                                     (2000, 50.0)])
def test_layer_step(cuda, ob, n, alpha):
    import torch

    q16, k, _ = inputs.config1(n, seed=1)
    v = inputs.values(1, n)
    q32 = np.frombuffer(q16.astype(np.uint16).tobytes(), dtype=np.float16).astype(np.float32)
    layer = cuda.SelectedKVLayer(n, alpha)
    out = layer(dev_u16(q16), _t(q32, torch.float32), dev_u16(k), dev_u16(v))
    sel = layer.selection()
    raw, ids, counts, kk = oracle_layer(ob, q16, q32, k, v, n, alpha)
    assert np.array_equal(host_u16(layer.scores), raw)
    assert sel.k == kk
    assert np.array_equal(layer.counts.cpu().numpy().astype(np.uint32), counts)
    if kk == 0:
        assert sel.status.code == 70  # the reference throws "zero selection" here
        assert float(out.abs().max()) == 0.0
        return
    assert sel.status.code == 0
    assert np.array_equal(layer.ids[:, :kk].cpu().numpy().astype(np.uint64), ids)
    count = layer.count
    payload = inputs.interleave(k, v, n).view(np.uint8)
    wk, wv, _ = ob.pack(ids, np.full(32, kk), [n - 1], np.arange(n, dtype=np.uint64), payload, count)
    gk = host_u16(layer.k_packed).reshape(count, 32, 128)[:kk]
    assert np.array_equal(gk, wk.reshape(count, 32, 128)[:kk])
    gv = host_u16(layer.v_packed).reshape(32, 128, count)[:, :, :kk]
    assert np.array_equal(gv, wv.reshape(32, 128, count)[:, :, :kk])
    want = ob.attention_compact(wk, wv, count, np.full(32, kk, dtype=np.uint32), q32)
    got = out.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got - want)) <= TOL * np.max(np.abs(want))


def test_layer_step_repeatable_in_graph(cuda, ob):
    """The layer step has no host round trip, so it captures into a CUDA
    graph; replays give identical bits."""
    import torch

    n, alpha = 4096, 10.0
    q16, k, _ = inputs.config1(n, seed=2)
    v = inputs.values(2, n)
    q32 = np.frombuffer(q16.astype(np.uint16).tobytes(), dtype=np.float16).astype(np.float32)
    layer = cuda.SelectedKVLayer(n, alpha)
    qd, q32d, kd, vd = dev_u16(q16), _t(q32, torch.float32), dev_u16(k), dev_u16(v)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        first = layer(qd, q32d, kd, vd).clone()
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        layer(qd, q32d, kd, vd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(layer.out, first)


@pytest.mark.parametrize("alpha", [5.0, 10.0])
def test_rehearsal_prefetch_step(cuda, ob, alpha):
    """configs[3] at N=4096: rehearsal query (x bf16, W_q bf16, RoPE at
    position N) -> F16 Q -> score the HBM keys -> select -> physical union ->
    stage the union's K|V rows from a pinned-host cold tier into HBM -> pack.
    From the GPU's F16 query on (the producer itself is checked to tolerance
    above), every stage is bit-exact against the oracle chain."""
    import torch

    n = 4096
    torch.manual_seed(11)
    x = torch.randn(4096, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(4096, 4096, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    _, q16 = cuda.rehearsal_query(x.cuda(), w.cuda(), n, 500000.0)
    q16h = host_u16(q16).reshape(-1)
    _, k, _ = inputs.config1(n, seed=3)
    v = inputs.values(3, n)
    rows = inputs.interleave(k, v, n)  # [n][2048] F16 bits: K[8][128] then V[8][128]
    cold = torch.from_numpy(rows.view(np.uint8).copy()).pin_memory()  # the pinned-host tier
    raw = cuda.score_full_gqa(q16.reshape(-1), [(dev_u16(k), n, 1024)])
    scaled = cuda.scale_scores(raw)
    sel = cuda.select_gqa_scores(scaled, 32, n, n, alpha, 0.2)
    torch.cuda.synchronize()
    wraw = ob.score(q16h, k, n, 1024)
    assert np.array_equal(host_u16(raw).reshape(-1), wraw.reshape(-1))
    wids, _, wk, _ = ob.select(ob.scale(wraw), 32, n, n, alpha, 0.2)
    assert sel.k == wk and wk > 0
    assert np.array_equal(sel.ids.cpu().numpy().astype(np.uint64), wids)
    sizes = torch.full((32,), sel.k, dtype=torch.int32, device="cuda")
    physical = cuda.gqa_physical_union(sel.ids_buffer, sizes, n)
    wphys = ob.union(wids, np.full(32, wk), n)
    assert np.array_equal(physical.cpu().numpy().astype(np.uint64), wphys)
    nphys = physical.numel()
    staged = torch.zeros(nphys * 4096, dtype=torch.uint8, device="cuda")
    cuda.stage_rows(cold.data_ptr(), physical, torch.tensor([nphys], dtype=torch.int32, device="cuda"), nphys, staged)
    torch.cuda.synchronize()
    assert np.array_equal(staged.cpu().numpy().reshape(nphys, 4096), rows.view(np.uint8).reshape(n, 4096)[wphys])
    count = max(32, (cuda.select_kmax(n, 0.2) + 31) // 32 * 32)
    kp = torch.empty(count * 4096, dtype=torch.int16, device="cuda")
    vp = torch.empty_like(kp)
    mask = torch.empty(32 * 64 * count, dtype=torch.float32, device="cuda")
    cuda.pack_gqa_workspace(sel.ids_buffer, sizes, [n], physical, staged, count, kp, vp, mask)
    payload = rows.view(np.uint8).reshape(n, 4096)[wphys].reshape(-1)
    wkp, wvp, wmask = ob.pack(wids, np.full(32, wk), [n], wphys, payload, count)
    assert np.array_equal(host_u16(kp), wkp) and np.array_equal(host_u16(vp), wvp)
    assert np.array_equal(mask.cpu().numpy(), wmask)


@pytest.mark.parametrize("n,alpha,seed", [(4096, 10.0, 5), (4096, 0.1, 6), (2000, 50.0, 7), (4103, 5.0, 8),
                                          (32768, 10.0, 9), (64, 50.0, 10)])
def test_prepare_select_equals_layer_step(cuda, ob, n, alpha, seed):
    """The split layer (hsb_layer_prepare scores the history [0, n-1);
    hsb_layer_select scores the current position n-1 in the selector) gives
    hsb_layer_step's bits: scores, k, ties, counts, IDs, packed K/V, output.
    The split's buffers start poisoned (0xff), so a read of the unscored
    current column would show; the whole result is also checked against the
    oracle.  Odd n puts the current position in the selector's tail loop."""
    import torch

    q16, k, _ = inputs.config1(n, seed=seed)
    v = inputs.values(seed, n)
    q32 = np.frombuffer(q16.astype(np.uint16).tobytes(), dtype=np.float16).astype(np.float32)
    qd, q32d, kd, vd = dev_u16(q16), _t(q32, torch.float32), dev_u16(k), dev_u16(v)
    whole = cuda.SelectedKVLayer(n, alpha)
    out_w = whole(qd, q32d, kd, vd).clone()
    sel_w = whole.selection()
    split = cuda.SelectedKVLayer(n, alpha)
    for t in (split.scores, split.workspace, split.ids, split.counts, split.k_packed, split.v_packed):
        t.view(torch.uint8).fill_(0xFF)
    split.prepare(qd, kd)
    out_s = split.select(qd, q32d, kd, vd)
    sel_s = split.selection()
    assert (sel_s.k, sel_s.boundary_tied_heads, sel_s.status.code) == (sel_w.k, sel_w.boundary_tied_heads,
                                                                        sel_w.status.code)
    assert torch.equal(split.scores, whole.scores)
    assert torch.equal(split.counts, whole.counts)
    kk = sel_w.k
    assert torch.equal(split.ids[:, :kk], whole.ids[:, :kk])
    count = whole.count
    assert torch.equal(split.k_packed.view(count, 32, 128)[:kk], whole.k_packed.view(count, 32, 128)[:kk])
    assert torch.equal(split.v_packed.view(32, 128, count)[:, :, :kk], whole.v_packed.view(32, 128, count)[:, :, :kk])
    assert torch.equal(out_s, out_w)
    raw, ids, counts, wk = oracle_layer(ob, q16, q32, k, v, n, alpha)
    assert np.array_equal(host_u16(split.scores), raw) and kk == wk


@pytest.mark.parametrize("where", ["head0", "other"])
def test_select_current_nonfinite(cuda, where):
    """A non-finite score at the current position raises the reference's
    error in the split as in the whole step: head 0 -> nonfinite head0 score
    (22), any other head -> nonfinite GQA score (24)."""
    import torch

    n = 4096
    q16, k, _ = inputs.config1(n, seed=12)
    v = inputs.values(12, n)
    kk = k.copy().reshape(n, 8, 128)
    kk[n - 1, 0 if where == "head0" else 5, 3] = 0x7C00  # +inf in the current position's key row
    q32 = np.frombuffer(q16.astype(np.uint16).tobytes(), dtype=np.float16).astype(np.float32)
    qd, q32d, kd, vd = dev_u16(q16), _t(q32, torch.float32), dev_u16(kk.reshape(-1)), dev_u16(v)
    whole = cuda.SelectedKVLayer(n, 5.0)
    whole(qd, q32d, kd, vd)
    split = cuda.SelectedKVLayer(n, 5.0)
    split.prepare(qd, kd)
    split.select(qd, q32d, kd, vd)
    a, b = whole.selection(), split.selection()
    assert a.status.code == b.status.code == (22 if where == "head0" else 24)
    assert a.status.index == b.status.index
