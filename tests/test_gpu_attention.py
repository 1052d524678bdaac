"""Stage 4 on the GPU: attention over the packed workspace (mask or per-head
lengths) and dense decode attention, against the double-precision oracle.
Tolerance: max relative error 2e-3."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from conftest import dev_u16

pytestmark = pytest.mark.gpu
TOL = 2e-3


def rel_err(got, want) -> float:
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def _t(a, dtype):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to("cuda")


def packed_case(seed: int, n: int, kk: int, count: int):
    rng = np.random.default_rng(seed)
    q, k, _ = inputs.config1(n, seed=seed)
    v = inputs.values(seed, n)
    ids = np.stack([np.sort(rng.permutation(n)[:kk])[::-1] for _ in range(32)]).astype(np.uint64)
    q32 = inputs.normals(seed, 4096, stream=9).astype(np.float32)
    payload = inputs.interleave(k, v, n).view(np.uint8)
    return ids, payload, q32


@pytest.mark.parametrize("n,kk,count", [(4096, 819, 832), (1000, 5, 32), (600, 300, 6560 // 20)])
def test_packed_with_mask(cuda, ob, n, kk, count):
    import torch

    ids, payload, q32 = packed_case(n, n, kk, count)
    sizes = np.full(32, kk)
    positions = [n - 1]
    wk, wv, wmask = ob.pack(ids, sizes, positions, np.arange(n, dtype=np.uint64), payload, count)
    want = ob.attention_packed(wk, wv, wmask, count, 64, q32)
    out = cuda.attention_packed(_t(q32, torch.float32), dev_u16(wk), dev_u16(wv), count,
                                mask=_t(wmask, torch.float32), qpad=64)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy().astype(np.float64), want) < TOL


@pytest.mark.parametrize("lengths", [[819] * 32, [1] * 32, list(range(1, 33)), [0] + [7] * 31])
def test_packed_with_lengths(cuda, ob, lengths):
    import torch

    n, count = 4096, 832
    ids, payload, q32 = packed_case(5, n, 819, count)
    sizes = np.array(lengths)
    wk, wv, _ = ob.pack(ids, np.maximum(sizes, 1), [n - 1], np.arange(n, dtype=np.uint64), payload, count)
    want = ob.attention_compact(wk, wv, count, sizes, q32)
    out = cuda.attention_packed(_t(q32, torch.float32), dev_u16(wk), dev_u16(wv), count,
                                sizes=_t(sizes, torch.int32), sizes_stride=1)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    assert rel_err(got, want) < TOL
    if lengths[0] == 0:
        assert np.all(got[0] == 0.0)


@pytest.mark.parametrize("n,stride", [(4096, 1024), (1500, 2048), (32768, 1024), (77, 1024)])
def test_dense(cuda, ob, n, stride):
    import torch

    q, k, _ = inputs.config1(n, seed=21)
    v = inputs.values(21, n)
    q32 = inputs.normals(21, 4096, stream=9).astype(np.float32)
    if stride == 2048:
        rows = inputs.interleave(k, v, n)
        dev = dev_u16(rows)
        kd, vd = dev, dev[1024:]
        want = ob.attention_dense(rows, rows[1024:], n, 2048, q32)
    else:
        kd, vd = dev_u16(k), dev_u16(v)
        want = ob.attention_dense(k, v, n, 1024, q32)
    out = cuda.attention_dense(_t(q32, torch.float32), kd, vd, n, stride)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy().astype(np.float64), want) < TOL


@pytest.mark.parametrize("factor,tol", [(1.0, 1e-4), (30.0, TOL), (1e5, TOL), (1e-4, TOL)])
def test_dense_query_range(cuda, ob, factor, tol):
    """The dense kernel's tensor-core path carries Q as F16 hi/lo halves after
    a power-of-two scale per KV head: queries far outside the F16 range (1e5)
    or near its subnormals (1e-4) keep their accuracy, and at unit scale the
    result stays near FP32 (1e-4, twenty times inside the stage tolerance)."""
    import torch

    n = 4096
    _, k, _ = inputs.config1(n, seed=23)
    v = inputs.values(23, n)
    q32 = (inputs.normals(23, 4096, stream=9) * factor).astype(np.float32)
    q32[5 * 128 + 17] *= 8.0  # one channel of one head well above the rest of its KV group
    want = ob.attention_dense(k, v, n, 1024, q32)
    out = cuda.attention_dense(_t(q32, torch.float32), dev_u16(k), dev_u16(v), n, 1024)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert rel_err(got, want) < tol
