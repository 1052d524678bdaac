"""Stage 3 parity on the GPU: physical union, pack (reference layout incl.
mask and zero padding), prefetch-map gather and HBM-cache gather, all
bit-exact against the reference's digests and the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from conftest import dev_u16, host_u16

pytestmark = pytest.mark.gpu


def _t(a, dtype):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to("cuda")


def gpu_pack(hsb, ids, sizes, positions, physical, payload, count):
    import torch

    qpad = (len(positions) + 63) // 64 * 64
    k = torch.empty(count * 4096, dtype=torch.int16, device="cuda")
    v = torch.empty_like(k)
    mask = torch.empty(count * qpad * 32, dtype=torch.float32, device="cuda")
    hsb.pack_gqa_workspace(_t(ids.astype(np.int64), torch.int32), _t(np.asarray(sizes, np.int64), torch.int32),
                           _t(np.asarray(positions, np.int64), torch.int64),
                           _t(np.asarray(physical, np.int64), torch.int32),
                           torch.from_numpy(np.ascontiguousarray(payload)).to("cuda"), count, k, v, mask)
    torch.cuda.synchronize()
    return host_u16(k), host_u16(v), mask.cpu().numpy()


def test_pack_known_answers(cuda, ob):
    ids = np.tile(np.array([8, 12], dtype=np.uint64), (32, 1))
    ids[4] = [12, 8]
    raw = np.zeros(4096, dtype=np.uint16)
    for t in range(2):
        for h in range(8):
            for d in range(128):
                raw[t * 2048 + h * 128 + d] = 1000 * t + 100 * h + d
                raw[t * 2048 + 1024 + h * 128 + d] = 5000 + 1000 * t + 100 * h + d
    payload = raw.view(np.uint8)
    got = gpu_pack(cuda, ids, [2] * 32, [10, 12], [8, 12], payload, 32)
    want = ob.pack(ids, [2] * 32, [10, 12], np.array([8, 12], dtype=np.uint64), payload, 32)
    for g, w in zip(got, want):
        assert np.array_equal(g.view(np.uint8), w.view(np.uint8))
    bad = np.vstack([np.array([[13, 0]], dtype=np.uint64), ids[1:]])
    with pytest.raises(cuda.InvalidArgument) as e:
        gpu_pack(cuda, bad, [1] + [2] * 31, [12], [8, 12], payload, 32)
    assert e.value.status == 43 and str(e.value) == "future or missing selected KV"


def test_pack_and_union_golden(cuda, golden):
    import torch
    from golden.make_golden import pack_case

    g = golden("pack_trials.npz")
    for i, name in enumerate(g["names"].tolist()):
        ids, sizes, positions, rows, payload, slots = pack_case(int(name[1:]))
        k, v, mask = gpu_pack(cuda, ids, sizes, positions, rows, payload, slots)
        assert inputs.digest(k) == g["k_digest"][i]
        assert inputs.digest(v) == g["v_digest"][i]
        assert inputs.digest(mask) == g["mask_digest"][i]
        u = cuda.gqa_physical_union(_t(ids.astype(np.int64), torch.int32), _t(sizes.astype(np.int64), torch.int32),
                                    len(rows))
        assert inputs.digest(u.cpu().numpy().astype(np.uint64)) == g["union_digest"][i]


def test_pack_errors(cuda):
    ids = np.tile(np.array([0, 1], dtype=np.uint64), (32, 1))
    payload = np.zeros(2 * 4096, dtype=np.uint8)
    with pytest.raises(cuda.InvalidArgument) as e:  # duplicate physical position
        gpu_pack(cuda, ids, [2] * 32, [5], [1, 1], payload, 32)
    assert e.value.status == 41
    with pytest.raises(cuda.InvalidArgument) as e:  # empty head
        gpu_pack(cuda, ids, [2] * 5 + [0] + [2] * 26, [5], [0, 1], payload, 32)
    assert e.value.status == 42 and str(e.value) == "per-head selection exceeds slots"
    with pytest.raises(cuda.InvalidArgument) as e:  # head larger than count
        gpu_pack(cuda, np.tile(np.arange(40, dtype=np.uint64), (32, 1)), [40] * 32, [50], np.arange(40),
                 np.zeros(40 * 4096, dtype=np.uint8), 32)
    assert e.value.status == 42
    with pytest.raises(cuda.InvalidArgument) as e:  # shape: payload size mismatch
        gpu_pack(cuda, ids, [2] * 32, [5], [0, 1], np.zeros(4096, dtype=np.uint8), 32)
    assert e.value.status == 40


def test_union_duplicates(cuda):
    import torch

    ids = np.zeros((32, 3), dtype=np.int64)
    ids[:, 0], ids[:, 1] = 1, 2
    sizes = np.full(32, 2)
    u = cuda.gqa_physical_union(_t(ids, torch.int32), _t(sizes, torch.int32), 5)
    assert u.cpu().tolist() == [1, 2]
    ids[31, 2] = 1
    sizes[31] = 3
    with pytest.raises(cuda.InvalidArgument):
        cuda.gqa_physical_union(_t(ids, torch.int32), _t(sizes, torch.int32), 5)
    with pytest.raises(cuda.InvalidArgument):
        cuda.gqa_physical_union(_t(ids, torch.int32), _t(np.full(32, 2), torch.int32), 2)


@pytest.mark.parametrize("visible", [5, 32768, 49152, 49153, 66048])
def test_union_paths(cuda, visible):
    """Both union shapes (membership words in shared memory up to 49152
    positions, in the global workspace past that, up to the reference's
    66048-position bound) give the sorted set of every head's IDs."""
    import torch

    rng = np.random.default_rng(visible)
    k = min(visible, 700)
    sizes = rng.integers(0, k + 1, 32)
    ids = np.zeros((32, k), dtype=np.int64)
    for h in range(32):
        ids[h, :sizes[h]] = rng.choice(visible, sizes[h], replace=False)
    want = np.unique(np.concatenate([ids[h, :sizes[h]] for h in range(32)]))
    u = cuda.gqa_physical_union(_t(ids, torch.int32), _t(sizes, torch.int32), visible)
    assert u.cpu().numpy().astype(np.int64).tolist() == want.tolist()


@pytest.mark.parametrize("count", [32, 37, 200])
def test_gather_map_vs_oracle(cuda, ob, count):
    import torch

    rng = np.random.default_rng(count)
    prows, mrows = 50, 20
    pre = rng.integers(0, 1 << 16, prows * 2048, dtype=np.uint32).astype(np.uint16)
    mis = rng.integers(0, 1 << 16, mrows * 2048, dtype=np.uint32).astype(np.uint16)
    row_map = rng.integers(-1 - mrows, prows, size=32 * count).astype(np.int32)
    k = torch.empty(count * 4096, dtype=torch.int16, device="cuda")
    v = torch.empty_like(k)
    cuda.gather_map(dev_u16(pre), prows, dev_u16(mis), mrows, _t(row_map, torch.int32), count, k, v)
    torch.cuda.synchronize()
    wk, wv = ob.gather_map(pre, prows, mis, mrows, row_map, count)
    assert np.array_equal(host_u16(k), wk) and np.array_equal(host_u16(v), wv)
    bad = row_map.copy()
    bad[5] = prows
    with pytest.raises(cuda.HsbError) as e:
        cuda.gather_map(dev_u16(pre), prows, dev_u16(mis), mrows, _t(bad, torch.int32), count, k, v)
    assert e.value.status == 51


@pytest.mark.parametrize("n,kk,stride", [(4096, 819, 1024), (1000, 37, 2048), (300, 300, 1024)])
def test_gather_cache_vs_pack(cuda, ob, n, kk, stride):
    """Gathering straight from an HBM cache gives the reference pack layout."""
    import torch

    rng = np.random.default_rng(n)
    q, k, _ = inputs.config1(n, seed=11)
    v = inputs.values(11, n)
    if stride == 2048:
        kc = inputs.interleave(k, v, n)
        vc_off = 1024
        cache = dev_u16(kc)
        kdev, vdev = cache, cache[vc_off:]
    else:
        kdev, vdev = dev_u16(k), dev_u16(v)
    ids = np.stack([rng.permutation(n)[:kk] for _ in range(32)]).astype(np.uint64)
    count = (kk + 31) // 32 * 32
    sizes = np.full(32, kk)
    kout = torch.empty(count * 4096, dtype=torch.int16, device="cuda")
    vout = torch.empty_like(kout)
    cuda.gather_cache(_t(ids.astype(np.int64), torch.int32), _t(sizes, torch.int32), 1, kdev, vdev, stride, n,
                      count, kout, vout, zero_padding=True)
    torch.cuda.synchronize()
    physical = np.arange(n, dtype=np.uint64)
    payload = inputs.interleave(k, v, n).view(np.uint8)
    wk, wv, _ = ob.pack(ids, sizes, [n - 1], physical, payload, count)
    assert np.array_equal(host_u16(kout), wk) and np.array_equal(host_u16(vout), wv)


def test_stage_rows_from_pinned_host(cuda):
    """Cold tier: rows read by the GPU straight from mapped pinned memory."""
    import torch

    n = 512
    rows = torch.randint(0, 255, (n * 4096,), dtype=torch.uint8).pin_memory()
    physical = torch.tensor([3, 7, 100, 511, 0], dtype=torch.int32, device="cuda")
    count = torch.tensor([5], dtype=torch.int32, device="cuda")
    dst = torch.zeros(8 * 4096, dtype=torch.uint8, device="cuda")
    cuda.stage_rows(rows.data_ptr(), physical, count, 8, dst)
    torch.cuda.synchronize()
    want = rows.view(n, 4096)[[3, 7, 100, 511, 0]]
    assert torch.equal(dst.view(8, 4096)[:5].cpu(), want)
    assert int(dst.view(8, 4096)[5:].sum()) == 0
