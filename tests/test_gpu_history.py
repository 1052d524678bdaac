"""The decode history on the GPU (hsb_history_*: FullGqaRuntimePolicy's
hot/cold scoring and prepare -> select -> fetch, policy/full_gqa_runtime.cpp:
418-690) against the oracle: history scores over hot-pool and cold-K runs,
the payload cover and its cold positions, the final selection with the
current token, and the packed K/V of the fetch -- bit for bit, with and
without a prepared history, for two placements; plus the protocol's
rejections."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from oracle import binding as ob

pytestmark = pytest.mark.gpu

PROMPT, GEN, CAP, ALPHA = 3968, 128, 4096, 5.0


def _rows(seed: int, n: int) -> np.ndarray:
    """Token-major K||V rows [n][2048] (F16 bits); K ~ N(0,1) with heavy
    rows x4, V ~ N(0,1)."""
    k = inputs.normals(seed, n * 1024, stream=2).reshape(n, 1024)
    k[inputs.heavy_rows(seed, n)] *= 4.0
    rows = np.empty((n, 2048), dtype=np.uint16)
    rows[:, :1024] = inputs.f16_bits(k)
    rows[:, 1024:] = inputs.values(seed, n).reshape(n, 1024)
    return rows


def _dev(a, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def _oracle_step(rows, q16, position, slots):
    """Reference semantics of one step: cover of [0, position), selection of
    [0, position] (full_gqa_runtime.cpp:299-344, 549-585)."""
    raw_hist = np.zeros((32, CAP), dtype=np.uint16)
    raw_hist[:, :position] = ob.score(q16, rows[:position, :1024].reshape(-1), position, 1024)
    per_head, physical = ob.prefetch_cover(raw_hist, CAP, position, ALPHA)
    cold = np.array([p for p in physical if slots[int(p)] < 0], dtype=np.uint64)
    raw = raw_hist.copy()
    raw[:, :position + 1] = ob.score(q16, rows[:position + 1, :1024].reshape(-1), position + 1, 1024)
    ids, counts, k, tied = ob.select(ob.scale(raw), 32, CAP, position + 1, ALPHA, 0.2)
    return per_head.shape[1], cold, ids, counts, k, tied


@pytest.mark.parametrize("beta", [1.0, 0.25])
def test_history_protocol_matches_oracle(cuda, beta):
    import torch
    import hillserve_b200 as hsb

    hist = hsb.History(2, CAP, PROMPT, GEN, beta=beta, alpha=ALPHA)
    slots = hist.slots
    assert hist.cold_rows == int((slots[:PROMPT] < 0).sum()) > 0
    layers = [_rows(100 + l, PROMPT + 4) for l in range(2)]
    for l in range(2):
        hist.append(l, 0, _dev(layers[l][:PROMPT], torch.int16))
    for step in range(3):
        position = PROMPT + step
        for l in range(2):
            rows = layers[l]
            q16 = inputs.f16_bits(inputs.normals(1000 * l + step, 4096, stream=1)).reshape(32, 128)
            bound, cold, ids, counts, k, tied = _oracle_step(rows, q16.reshape(-1), position, slots)
            qd = _dev(q16, torch.int16)
            prepared = not (l == 1 and step == 1)  # one select without a prepared history
            staged_ids = None
            if prepared:
                hist.prepare_history(l, position, qd)
                got_cold, got_bound = hist.cover(l)
                assert got_bound == bound
                assert np.array_equal(got_cold.cpu().numpy().astype(np.uint64), cold)
                staged_ids = got_cold
            else:
                staged_ids = _dev(np.array([p for p in range(position) if slots[p] < 0], dtype=np.int32))
            hist.append(l, position, _dev(rows[position:position + 1], torch.int16))
            gids, gcounts, res = hist.select(l, position, qd)
            r = res.cpu().numpy()
            assert (r[0], r[1], r[2]) == (k, tied, 0)
            assert np.array_equal(gcounts.cpu().numpy().astype(np.uint32), counts)
            assert np.array_equal(gids[:, :k].cpu().numpy().astype(np.uint64), ids)
            staged = staged_ids.cpu().numpy().astype(np.int64)
            count = (k + 31) // 32 * 32
            kp, vp, _ = hist.fetch(l, gids, res, staged_ids, _dev(rows[staged], torch.int16), count)
            sel = ids.astype(np.int64)
            kk = rows[sel, :1024].reshape(32, k, 8, 128)[np.arange(32), :, np.arange(32) // 4, :]  # [32][k][128]
            vv = rows[sel, 1024:].reshape(32, k, 8, 128)[np.arange(32), :, np.arange(32) // 4, :]
            kp = kp.cpu().numpy().view(np.uint16)
            vp = vp.cpu().numpy().view(np.uint16)
            assert np.array_equal(kp[:k], kk.transpose(1, 0, 2))
            assert np.array_equal(vp[:, :, :k], vv.transpose(0, 2, 1))
            assert not kp[k:].any() and not vp[:, :, k:].any()
    hist.close()


def test_score_history_runs_equal_full_scorer(cuda):
    """hsb_score_history over a fragmented map (64-token blocks alternating
    between pool and cold store, out of order in the pool) equals scoring
    the token-major K."""
    import torch
    import hillserve_b200 as hsb

    n = 2048
    rows = _rows(7, n)
    q16 = inputs.f16_bits(inputs.normals(3, 4096, stream=1))
    blocks = np.arange(n // 64)
    hot_blocks = blocks[blocks % 3 != 1][::-1]  # reversed order in the pool
    row_of = np.full(n, -1, dtype=np.int64)
    pool_rows, cold_rows = [], []
    for b in hot_blocks:
        for t in range(b * 64, b * 64 + 64):
            row_of[t] = len(pool_rows)
            pool_rows.append(rows[t])
    for b in blocks[blocks % 3 == 1]:
        for t in range(b * 64, b * 64 + 64):
            row_of[t] = -2 - len(cold_rows)
            cold_rows.append(rows[t, :1024])
    pool = _dev(np.stack(pool_rows), torch.int16)
    cold = _dev(np.stack(cold_rows), torch.int16)
    got = hsb.score_history(_dev(q16, torch.int16), pool, cold, row_of, n)
    torch.cuda.synchronize()
    want = ob.score(q16, rows[:, :1024].reshape(-1), n, 1024)
    assert np.array_equal(got.cpu().numpy().view(np.uint16), want)
    row_of[100] = -1
    with pytest.raises(hsb.HsbError):
        hsb.score_history(_dev(q16, torch.int16), pool, cold, row_of, n)


def test_history_protocol_rejections(cuda):
    import torch
    import hillserve_b200 as hsb

    hist = hsb.History(3, CAP, PROMPT, GEN, beta=1.0, alpha=ALPHA)
    rows = _rows(5, PROMPT + 2)
    for l in range(3):
        hist.append(l, 0, _dev(rows[:PROMPT], torch.int16))
    q = _dev(inputs.f16_bits(inputs.normals(1, 4096, stream=1)).reshape(32, 128), torch.int16)
    with pytest.raises(hsb.HsbError, match="incremental append range"):
        hist.append(0, PROMPT + 1, _dev(rows[:1], torch.int16))
    with pytest.raises(hsb.HsbError, match="exactly completed past positions"):
        hist.prepare_history(0, PROMPT - 1, q)
    with pytest.raises(hsb.HsbError, match="current KV append"):
        hist.select(0, PROMPT, q)
    hist.prepare_history(0, PROMPT, q)
    with pytest.raises(hsb.HsbError, match="at most two"):
        hist.prepare_history(0, PROMPT, q)
    hist.prepare_history(1, PROMPT, q)
    with pytest.raises(hsb.HsbError, match="at most two"):
        hist.prepare_history(2, PROMPT, q)
    with pytest.raises(hsb.HsbError, match="only its current-token append"):
        hist.append(0, PROMPT, _dev(rows[PROMPT:PROMPT + 2], torch.int16))
    hist.append(0, PROMPT, _dev(rows[PROMPT:PROMPT + 1], torch.int16))
    other = _dev(inputs.f16_bits(inputs.normals(2, 4096, stream=1)).reshape(32, 128), torch.int16)
    _, _, res = hist.select(0, PROMPT, other)  # not the prepared query
    assert int(res[2].item()) == 103
    with pytest.raises(hsb.HsbError, match="duplicate/backwards"):
        hist.select(0, PROMPT, q)
    # a selected cold position that was not staged
    hist.append(1, PROMPT, _dev(rows[PROMPT:PROMPT + 1], torch.int16))
    ids, counts, res = hist.select(1, PROMPT, q)
    k = int(res[0].item())
    sel = ids[:, :k].cpu().numpy()
    cold_selected = [p for p in np.unique(sel) if hist.slots[p] < 0]
    if cold_selected:
        _, _, st = hist.fetch(1, ids, res, None, None, 32 * ((k + 31) // 32), check=False)
        torch.cuda.synchronize()
        assert int(st[0].item()) == 52  # HSB_E_MAP_MISS
    hist.close()


@pytest.mark.parametrize("i", [0, 1, 2, 3, 4])
def test_history_matches_reference_runtime(cuda, i):
    """The GPU decode history against the reference's own runtime outputs
    (tests/golden/runtime_decode.npz, made by running FullGqaRuntimePolicy
    from the reference sources): per step the cover's bound and its cold
    positions (the rows the runtime reads from the cold tier) after
    prepare, and the final per-head selection after the current token's
    append -- bit for bit."""
    import sys
    from pathlib import Path

    import torch
    import hillserve_b200 as hsb

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden as mg

    fx = np.load(Path(__file__).resolve().parent / "golden" / "runtime_decode.npz", allow_pickle=False)
    seed, cap, prompt, steps, layer, beta, alpha = [t(x) for t, x in zip((int,) * 5 + (float, float),
                                                                          mg.RUNTIME_CASES[i])]
    rows = mg.runtime_rows(seed, cap)
    q = mg.runtime_queries(seed, steps)
    hist = hsb.History(layer + 1, cap, prompt, steps, beta=beta, alpha=alpha)
    hist.append(layer, 0, _dev(rows[:prompt], torch.int16))
    for s in range(steps):
        pos = prompt + s
        qd = _dev(q[s].astype(np.float16).view(np.uint16).reshape(32, 128), torch.int16)
        hist.prepare_history(layer, pos, qd)
        got_cold, got_bound = hist.cover(layer)
        assert got_bound == int(fx[f"c{i}_bound"][s])
        n = int(fx[f"c{i}_nphysical"][s])
        phys = fx[f"c{i}_physical"][s][:n].astype(np.int64)
        want_cold = phys[fx[f"c{i}_cold"][s][:n].astype(bool)]
        assert np.array_equal(got_cold.cpu().numpy().astype(np.int64), want_cold)
        hist.append(layer, pos, _dev(rows[pos:pos + 1], torch.int16))
        gids, _, res = hist.select(layer, pos, qd)
        k = int(fx[f"c{i}_k"][s])
        r = res.cpu().numpy()
        assert r[0] == k and r[2] == 0, r
        assert np.array_equal(gids[:, :k].cpu().numpy().astype(np.uint32), fx[f"c{i}_final"][s][:, :k])
        staged = got_cold.cpu().numpy().astype(np.int64)
        hist.fetch(layer, gids, res, got_cold, _dev(rows[staged], torch.int16), (k + 31) // 32 * 32)
    hist.close()
