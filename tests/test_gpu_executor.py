"""The model-facing decode step (hsb_executor_*, runtime/gqa_executor.cpp:
149-249 on the GPU): the model's current KV tensor appended to the HBM cache
bit for bit with its non-finite check, the rehearsal's F16 rounding with the
reference's rule and errors, and a decode layer -- sparse (selection by the
rehearsal, attention over live slots with the layer's own query) and dense
-- against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
import shard_oracle as so
from oracle import binding as ob

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _current(seed: int, n: int) -> np.ndarray:
    """[n][8][256] F16 bits: K (heavy rows x4) | V per KV head."""
    k = inputs.normals(seed, n * 1024, stream=2).reshape(n, 8, 128)
    k[inputs.heavy_rows(seed, n)] *= 4.0
    cur = np.empty((n, 8, 256), dtype=np.uint16)
    cur[:, :, :128] = inputs.f16_bits(k)
    cur[:, :, 128:] = inputs.values(seed, n).reshape(n, 8, 128)
    return cur


def _dev(a, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t.view(dtype) if dtype is not None else t).cuda()


def test_append_layout_and_nonfinite(cuda):
    import torch
    import hillserve_b200 as hsb

    ex = hsb.DecodeExecutor(1, 1024)
    cur = _current(3, 300)
    ex.append(0, _dev(cur, torch.int16))
    torch.cuda.synchronize()
    rows = ex.cache[0][:300].cpu().numpy().view(np.uint16)
    assert np.array_equal(rows[:, :1024].reshape(300, 8, 128), cur[:, :, :128])
    assert np.array_equal(rows[:, 1024:].reshape(300, 8, 128), cur[:, :, 128:])
    assert not ex.status.any()
    bad = _current(4, 5)
    bad[3, 6, 200] = 0x7C00  # +inf in V
    ex.append(0, _dev(bad, torch.int16))
    torch.cuda.synchronize()
    assert ex.status.cpu().numpy().tolist() == [111, 3]


def test_rehearsal_rounding(cuda):
    import torch
    import hillserve_b200 as hsb

    x = (inputs.normals(9, 4096, stream=5) * 1000).astype(np.float32)
    x[7] = 65519.0   # rounds to 65504
    x[8] = -6e-8     # subnormal range
    q16 = torch.empty(4096, dtype=torch.int16, device="cuda")
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert hsb.lib().hsb_executor_query(_dev(x).data_ptr(), q16.data_ptr(), st.data_ptr(), None) == 0
    torch.cuda.synchronize()
    want = np.array([ob.half_bits(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(q16.cpu().numpy().view(np.uint16), want) and not st.any()
    y = x.copy()
    y[11] = 70000.0  # F16 overflow
    y[40] = np.nan
    st.zero_()
    hsb.lib().hsb_executor_query(_dev(y).data_ptr(), q16.data_ptr(), st.data_ptr(), None)
    torch.cuda.synchronize()
    assert st.cpu().numpy().tolist() == [113, 11]


@pytest.mark.parametrize("alpha", [5.0, 0.1])
def test_decode_layers_match_oracle(cuda, alpha):
    import torch
    import hillserve_b200 as hsb

    n = 2048
    cap = 2112
    ex = hsb.DecodeExecutor(3, cap, alpha=alpha)
    cur = _current(11, n + 1)
    for layer in range(3):
        ex.append(layer, _dev(cur[:n], torch.int16))  # the prompt, as prefill appends it
    rehearsal = inputs.normals(21, 4096, stream=1).astype(np.float32).reshape(32, 128)
    q = inputs.normals(22, 4096, stream=1).astype(np.float32).reshape(32, 128)
    q16 = np.array([ob.half_bits(float(v)) for v in rehearsal.reshape(-1)], dtype=np.uint16)
    k = cur[:, :, :128].copy()
    v = cur[:, :, 128:].copy()
    # sparse layer 2: selection by the rehearsal, attention with q
    out = ex.decode_layer(2, _dev(cur[n:n + 1], torch.int16), _dev(rehearsal), _dev(q))
    torch.cuda.synchronize()
    ids, counts, kk, tied, want, _ = so.unsharded(ob, q16, q, k, v, n + 1, alpha)
    res = ex.result.cpu().numpy()
    assert (res[0], res[1], res[2]) == (kk, tied, 0)
    assert np.array_equal(ex.ids[:, :kk].cpu().numpy().astype(np.uint64), ids)
    got = out.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got - want)) <= TOL * np.max(np.abs(want))
    # dense layer 0: every position
    out0 = ex.decode_layer(0, _dev(cur[n:n + 1], torch.int16), _dev(rehearsal), _dev(q))
    torch.cuda.synchronize()
    kf = k.view(np.float16).astype(np.float64)
    vf = v.view(np.float16).astype(np.float64)
    dense = np.stack([so.attention(q[h], kf[:, h // 4, :], vf[:, h // 4, :]) for h in range(32)])
    assert np.max(np.abs(out0.cpu().numpy() - dense)) <= TOL * np.max(np.abs(dense))
    assert not ex.status.any()
