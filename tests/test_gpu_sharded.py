"""KV-head-sharded layer on one GPU: W shards (W = 1, 2, 4, 8) run through the
real kernels in one process, with the three exchanges of a sharded step done
by concatenation, against the unsharded reference path.  Bit-exact: scores,
k, counts, per-head IDs, packed K/V rows; attention within 2e-3."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
import shard_oracle as so

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _sequences(n: int, batch: int, seed: int):
    qs, ks, vs = [], [], []
    for b in range(batch):
        q16, k, _ = inputs.config1(n, seed=seed + b)
        qs.append(q16.reshape(32, 128))
        ks.append(k.reshape(n, 8, 128))
        vs.append(inputs.values(seed + b, n).reshape(n, 8, 128))
    return np.stack(qs), np.stack(ks), np.stack(vs)


def _run_shards(cuda, world, n, batch, alpha, q16, q32, k, v):
    import torch
    from hillserve_b200 import sharded as sh

    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()  # noqa: E731
    q16t = dev(q16.view(np.int16), torch.int16)
    q32t = dev(q32, torch.float32)
    kt = dev(k.view(np.int16), torch.int16)
    vt = dev(v.view(np.int16), torch.int16)
    layers = [sh.KVHeadShardedLayer(n, batch, world, r, alpha=alpha) for r in range(world)]
    qs16 = [sh.shard_queries(q16t, world, r) for r in range(world)]
    qs32 = [sh.shard_queries(q32t, world, r) for r in range(world)]
    kss = [sh.shard_rows(kt, world, r) for r in range(world)]
    vss = [sh.shard_rows(vt, world, r) for r in range(world)]
    s = torch.cuda.current_stream().cuda_stream
    for r, layer in enumerate(layers):
        layer.score(qs16[r], kss[r], s)
    layers[0].threshold(s)
    for layer in layers[1:]:
        layer.thr.copy_(layers[0].thr)  # broadcast
    for layer in layers:
        layer.count_heads(s)
    records = torch.cat([layer.records for layer in layers], dim=1)  # all-gather in head order
    for r, layer in enumerate(layers):
        layer.records_all.copy_(records)
        layer.select(qs32[r], kss[r], vss[r], s)
    torch.cuda.synchronize()
    return layers


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("n,alpha", [(4096, 10.0), (4096, 0.1), (1024, 5.0)])
def test_sharded_layer_matches_unsharded(cuda, ob, world, n, alpha):
    batch = 3
    q16, k, v = _sequences(n, batch, seed=40 + world)
    q32 = q16.view(np.float16).astype(np.float32)
    layers = _run_shards(cuda, world, n, batch, alpha, q16, q32, k, v)
    h = 32 // world
    for b in range(batch):
        ids, counts, kk, tied, out, _ = so.unsharded(ob, q16[b], q32[b], k[b], v[b], n, alpha)
        raw = ob.score(q16[b].reshape(-1), k[b].reshape(-1), n, 1024)
        ties = 0
        for r, layer in enumerate(layers):
            res = layer.results[b].cpu().numpy()
            assert res[0] == kk, (r, res, kk)
            assert res[2] == (so.E_ZERO if kk == 0 else 0)
            ties += int(res[1])
            lo = h * r
            assert np.array_equal(layer.scores[b].cpu().numpy().view(np.uint16), raw[lo:lo + h])
            assert np.array_equal(layer.counts[b].cpu().numpy().astype(np.uint32), counts[lo:lo + h])
            got_out = layer.out[b].cpu().numpy().astype(np.float64)
            if kk == 0:
                assert np.all(got_out == 0.0)
                continue
            assert np.array_equal(layer.ids[b][:, :kk].cpu().numpy().astype(np.uint64), ids[lo:lo + h])
            want = out[lo:lo + h]
            assert np.max(np.abs(got_out - want)) <= TOL * np.max(np.abs(want))
            # packed K/V of this sequence
            kp = layer.k_packed[b].cpu().numpy().view(np.uint16).reshape(layer.count, h, 128)[:kk]
            vp = layer.v_packed[b].cpu().numpy().view(np.uint16).reshape(h, 128, layer.count)[:, :, :kk]
            sel = ids[lo:lo + h].astype(np.int64)
            kk_rows = k[b][sel, (np.arange(lo, lo + h) // 4)[:, None], :]  # [h][kk][128]
            vv_rows = v[b][sel, (np.arange(lo, lo + h) // 4)[:, None], :]
            assert np.array_equal(kp, kk_rows.transpose(1, 0, 2))
            assert np.array_equal(vp, vv_rows.transpose(0, 2, 1))
        assert ties == tied


def test_sharded_threshold_error_propagates(cuda, ob):
    """A non-finite head-0 score: every shard reports the reference's head-0
    error and leaves its output zero."""
    n, batch, world = 1024, 3, 2
    q16, k, v = _sequences(n, batch, seed=7)
    k = k.copy()
    k[1, 5, 0, :] = 0x7C00  # sequence 1: +inf in token 5's KV head 0 -> query head 0 score non-finite
    q32 = q16.view(np.float16).astype(np.float32)
    layers = _run_shards(cuda, world, n, batch, 10.0, q16, q32, k, v)
    for layer in layers:
        res = layer.results[1].cpu().numpy()
        assert res[2] == 22 and res[0] == 0
        assert float(layer.out[1].abs().max()) == 0.0
        for b in (0, 2):  # the other sequences of the batch are unaffected
            assert layer.results[b].cpu().numpy()[2] in (0, so.E_ZERO)


# ------------------------------------------------------------ peer memory
def _peer_step(cuda, n, batch, alpha, q16, q32, k, v, steps=2, graph=False):
    """One rank (world 1) through the peer-memory exchange kernels."""
    import torch
    from hillserve_b200 import sharded as sh

    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()  # noqa: E731
    q16t, q32t = dev(q16.view(np.int16), torch.int16), dev(q32, torch.float32)
    kt, vt = dev(k.view(np.int16), torch.int16), dev(v.view(np.int16), torch.int16)
    layer = sh.KVHeadShardedLayer(n, batch, 1, 0, alpha=alpha)
    ex = sh.PeerExchange(batch, 1, 0, wait_limit_ns=200_000_000)
    try:
        outs = []
        for _ in range(steps):  # the epoch advances every step
            out, res = layer.step_peer(q16t, q32t, kt, vt, ex)
            outs.append((out.clone(), res.clone()))
        if graph:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                layer.step_peer(q16t, q32t, kt, vt, ex)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                layer.step_peer(q16t, q32t, kt, vt, ex)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            out, res = ex.outputs, ex.results[0]
            outs.append((out.clone(), res.clone()))
            del g
        torch.cuda.synchronize()
        status = ex.status.cpu().numpy().copy()
        return outs, status
    finally:
        torch.cuda.synchronize()
        ex.close()


@pytest.mark.parametrize("n,alpha", [(4096, 10.0), (4096, 0.1)])
def test_peer_exchange_world1_matches_unsharded(cuda, ob, n, alpha):
    """World 1 through the mailbox kernels (threshold push, count + wait,
    select from the mailbox, finish): every step -- and graph replays, whose
    epochs come from the mailbox -- gives the unsharded reference's k,
    selections and outputs."""
    batch = 3
    q16, k, v = _sequences(n, batch, seed=90)
    q32 = q16.view(np.float16).astype(np.float32)
    outs, status = _peer_step(cuda, n, batch, alpha, q16, q32, k, v, steps=2, graph=True)
    assert status[0] == 0, status
    for out, res in outs:
        res = res.cpu().numpy()
        for b in range(batch):
            ids, counts, kk, tied, want, _ = so.unsharded(ob, q16[b], q32[b], k[b], v[b], n, alpha)
            assert res[b, 0] == kk and res[b, 1] == tied
            assert res[b, 2] == (so.E_ZERO if kk == 0 else 0)
            got = out[b].cpu().numpy().astype(np.float64)
            if kk == 0:
                assert np.all(got == 0.0)
            else:
                assert np.max(np.abs(got - want)) <= TOL * np.max(np.abs(want))
    for out, _ in outs[1:]:
        assert bool((out == outs[0][0]).all())


def test_peer_exchange_waits_run_out(cuda):
    """A peer that never arrives: the bounded waits of the exchange give up
    after the group's limit, write HSB_E_TIMEOUT (index = the rank waited
    for) into the mailbox's status word, and the kernels return -- the
    context stays usable.  Both 'ranks' are mailboxes on this GPU and only
    one side runs, so the flags they wait for are never set."""
    import ctypes as C
    import time

    import torch
    from hillserve_b200 import _capi

    lib = _capi.lib()
    batch, tokens, heads = 2, 256, 16
    lay = _capi.MailboxLayout()
    lib.hsb_mailbox_layout_of(batch, C.byref(lay))
    keys = torch.zeros(batch * heads * tokens, dtype=torch.int16, device="cuda")
    out = torch.zeros(batch * heads * 128, dtype=torch.float32, device="cuda")
    res = torch.zeros(batch * 4, dtype=torch.int32, device="cuda")
    for kernel in ("count", "finish"):
        mbs = []
        for _ in range(2):
            p = C.c_void_p()
            assert lib.hsb_mailbox_create(batch, C.byref(p), None) == 0
            mbs.append(p.value)
        g = _capi.PeerGroup()
        g.world, g.batch, g.wait_limit_ns = 2, batch, 200_000  # 200 us
        g.rank = 1 if kernel == "count" else 0
        g.mailbox[0], g.mailbox[1] = mbs[0], mbs[1]
        s = torch.cuda.current_stream().cuda_stream
        t0 = time.perf_counter()
        if kernel == "count":  # rank 1 waits for rank 0's thresholds
            rc = lib.hsb_exchange_count(keys.data_ptr(), heads, tokens, C.byref(g), s)
        else:  # rank 0 waits for rank 1's outputs
            rc = lib.hsb_exchange_finish(out.data_ptr(), res.data_ptr(), heads, C.byref(g), s)
        assert rc == 0, lib.hsb_last_error()
        own = mbs[g.rank]
        code = lib.hsb_status_check(C.c_void_p(own + lay.status), s)
        elapsed = time.perf_counter() - t0
        assert code == 4, (kernel, code)  # HSB_E_TIMEOUT
        word = torch.as_tensor(_Dev(own + lay.status), device="cuda").cpu().numpy()
        assert word[0] == 4 and word[1] == (0 if kernel == "count" else 1), word
        assert elapsed < 5.0
        torch.cuda.synchronize()  # the context is still usable
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
        for p in mbs:
            assert lib.hsb_mailbox_destroy(C.c_void_p(p)) == 0


class _Dev:
    """Two int32 words of device memory, as a torch view."""

    def __init__(self, ptr):
        self.__cuda_array_interface__ = {"shape": (2,), "typestr": "<i4", "data": (ptr, False), "version": 3,
                                         "strides": None}
