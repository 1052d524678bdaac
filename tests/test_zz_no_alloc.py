"""hsb_attention_packed_noalloc: the allocation-free attention entry point.

Its output must equal hsb_attention_packed's (same kernel, scratch in a static
device array instead of a caller workspace) within the attention tolerance,
on two calls in a row with different inputs -- the second call reuses the
scratch the first one left behind -- and the oracle's double-precision
attention over the same live slots.  Counts beyond the static scratch's slot
limit are rejected before any GPU work."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

TOL = 2e-3           # max relative error, as the other attention tests
MAX_SLOTS = 6592     # HSB_NOALLOC_MAX_SLOTS
E_WORKSPACE = 3


def rel_err(got, want) -> float:
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def _lib():
    from hillserve_b200 import _capi

    if not _capi.LIB_PATH.exists():
        from hillserve_b200 import build

        build.build()
    return _capi.lib()


def _case(torch, seed: int, count: int):
    """Packed K [count][32][128], V [32][128][count] (F16 bits), q F32 [32][128]
    and per-head live lengths <= count."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal(count * 4096).astype(np.float16).view(np.int16)
    v = rng.standard_normal(count * 4096).astype(np.float16).view(np.int16)
    q = rng.standard_normal(4096).astype(np.float32)
    sizes = rng.integers(1, count + 1, size=32).astype(np.int32)
    sizes[0] = count
    dev = lambda a: torch.from_numpy(a).to("cuda")  # noqa: E731
    return dev(q), dev(k), dev(v), dev(sizes)


def test_rejects_counts_beyond_the_static_scratch():
    lib = _lib()
    rc = lib.hsb_attention_packed_noalloc(None, None, None, MAX_SLOTS + 1, None, 0, None, 0, None, None)
    assert rc == E_WORKSPACE
    assert f"exceeds the {MAX_SLOTS}-slot limit" in lib.hsb_last_error().decode()


@pytest.mark.gpu
def test_matches_workspace_entry_on_two_calls_in_a_row(ob):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib()
    s = torch.cuda.current_stream().cuda_stream
    # Second call: more splits than the first, so it reads partials and
    # counters the first call left in the shared scratch.
    for seed, count in ((11, 1024), (12, MAX_SLOTS)):
        q, k, v, sizes = _case(torch, seed, count)
        ws = torch.empty(lib.hsb_attention_workspace_bytes(count), dtype=torch.uint8, device="cuda")
        want = torch.empty(4096, dtype=torch.float32, device="cuda")
        got = torch.full((4096,), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.hsb_attention_packed(q.data_ptr(), k.data_ptr(), v.data_ptr(), count, None, 0, sizes.data_ptr(), 1,
                                      want.data_ptr(), ws.data_ptr(), ws.numel(), s)
        assert rc == 0, lib.hsb_last_error()
        rc = lib.hsb_attention_packed_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), count, None, 0,
                                              sizes.data_ptr(), 1, got.data_ptr(), s)
        assert rc == 0, lib.hsb_last_error()
        torch.cuda.synchronize()
        w, g = want.cpu().numpy().astype(np.float64), got.cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(g))
        assert rel_err(g, w) <= TOL, (seed, count)
        # and the oracle's double-precision attention over the same live slots
        exact = ob.attention_compact(k.cpu().numpy().view(np.uint16), v.cpu().numpy().view(np.uint16), count,
                                     sizes.cpu().numpy().astype(np.uint32), q.cpu().numpy()).reshape(-1)
        assert rel_err(g, exact) <= TOL, (seed, count)


@pytest.mark.gpu
def test_calls_leave_device_memory_unchanged():
    """The promise itself: once the first call has resolved the scratch
    address, further calls take no device memory (a cudaMalloc of any size
    moves the device's free-memory figure by at least one 2 MiB page)."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib()
    s = torch.cuda.current_stream().cuda_stream
    q, k, v, sizes = _case(torch, 13, MAX_SLOTS)
    out = torch.empty(4096, dtype=torch.float32, device="cuda")
    call = lambda: lib.hsb_attention_packed_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), MAX_SLOTS,  # noqa: E731
                                                    None, 0, sizes.data_ptr(), 1, out.data_ptr(), s)
    assert call() == 0, lib.hsb_last_error()  # set-up: the scratch address of this context
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert call() == 0, lib.hsb_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert np.all(np.isfinite(out.cpu().numpy()))
