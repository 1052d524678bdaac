"""Cold-tier KV records on the GPU through the C-ABI: the encoder
(hsb_kv_records_encode) bit for bit against the oracle and the reference
store's own files (fixture), and the verifier (hsb_kv_records_verify) on
windows laid out by the read plan, against the oracle's walk of the
reference's validation loop -- clean reads, every kind of corruption, the
error order with and without validation groups, and out-of-window records;
plus a full-size encode -> verify round trip."""
from __future__ import annotations

import numpy as np
import pytest

import inputs
from oracle import binding as ob

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gpu_encode(payload: np.ndarray, count, nbytes, request, layer, first, stride=None):
    import torch
    import hillserve_b200 as hsb

    out = hsb.kv_records_encode(_dev(payload.reshape(-1)), count, nbytes, request, layer, first, payload_stride=stride)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("nbytes,stride,count", [(4096, 4096, 70), (4096, 4112, 33), (100, 100, 37),
                                                 (100, 104, 5), (4128, 4128, 9), (64, 72, 1000), (1, 1, 3)])
def test_encode_matches_oracle(cuda, nbytes, stride, count):
    payload = inputs.record_payload(nbytes + count, count, stride)
    got = _gpu_encode(payload, count, nbytes, 991, 7, 123, stride)
    want = ob.records_encode(payload, count, nbytes, 991, 7, 123, stride)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_encoded_file_equals_reference_store_file(cuda, case):
    from test_records import GOLDEN, _make_golden

    mg = _make_golden()
    request, layers, positions, nbytes, payloads = mg.record_case(case)

    def encode(rows, count, nb, req, layer, first):
        return _gpu_encode(rows, count, nb, req, layer, first)

    img = inputs.segment_image(request, layers, positions, nbytes, payloads, encode)
    assert inputs.digest(img) == str(np.load(GOLDEN)[f"file{case}_digest"])


def _windows(img: np.ndarray, ids, layer, positions, nbytes):
    """Reads the records of `ids` the way the runtime does: offset order,
    the bounded read plan, each window's bytes back to back in one buffer."""
    import hillserve_b200 as hsb

    stride = nbytes + 32
    offs = [4096 + (layer * positions + int(i)) * stride for i in ids]
    plan = hsb.kv_read_plan(offs, stride, img.nbytes)
    chunks, base, local = [], 0, []
    for (b, e, _, r0, r1) in plan:
        chunks.append(img[b:e])
        local += [base + offs[r] - b for r in range(r0, r1)]
        base += e - b
    window = np.concatenate(chunks)
    groups = np.array(hsb.kv_read_groups(plan, len(ids)), dtype=np.uint32)
    return window, np.array(local, dtype=np.uint64), groups


def _gpu_verify(window, offsets, positions, request, layer, nbytes, groups=None, out_rows=None, capacity=None):
    import torch
    import hillserve_b200 as hsb

    cap = len(offsets) if capacity is None else capacity
    out = torch.zeros((cap, nbytes), dtype=torch.uint8, device="cuda")
    st = hsb.kv_records_verify(_dev(window), _dev(offsets.astype(np.int64)), _dev(np.asarray(positions, np.int64)),
                               request, layer, nbytes, out,
                               groups=None if groups is None else _dev(groups.astype(np.int32)),
                               out_rows=None if out_rows is None else _dev(np.asarray(out_rows, np.int32)),
                               check=False)
    torch.cuda.synchronize()
    code, index = (int(x) for x in st.cpu().numpy())
    return code, index, out.cpu().numpy()


def _store(nbytes=4096, positions=300, layers=2, request=765):
    payloads = [inputs.record_payload(31 + l, positions, nbytes) for l in range(layers)]
    img = inputs.segment_image(request, layers, positions, nbytes, payloads, ob.records_encode)
    return img, payloads, request, positions


@pytest.mark.parametrize("nbytes", [4096, 100])
def test_verify_clean_windows(cuda, nbytes):
    img, payloads, request, positions = _store(nbytes)
    ids = np.sort(np.random.default_rng(nbytes).choice(positions, 97, replace=False)).astype(np.uint64)
    window, offsets, groups = _windows(img, ids, 1, positions, nbytes)
    rows = np.random.default_rng(1).permutation(len(ids))  # output rows in another order
    code, index, out = _gpu_verify(window, offsets, ids, request, 1, nbytes, groups, rows)
    assert (code, index) == (0, 0)
    assert np.array_equal(out[rows], payloads[1][ids.astype(np.int64)])
    ocode, _, oout = ob.records_verify(window, offsets, ids, request, 1, nbytes, groups, rows)
    assert ocode == 0 and np.array_equal(out, oout)


@pytest.mark.parametrize("flips", [
    [("payload", 5)], [("position", 5)], [("layer", 0)], [("request", 96)], [("version", 50)], [("digest", 7)],
    [("payload", 9), ("position", 10)],   # same group of four: identity first with groups, checksum first without
    [("payload", 12), ("position", 40)], [("digest", 3), ("payload", 2)],
])
def test_verify_rejects_like_reference_loop(cuda, flips):
    img, payloads, request, positions = _store(4096)
    ids = np.sort(np.random.default_rng(3).choice(positions, 97, replace=False)).astype(np.uint64)
    window, offsets, groups = _windows(img, ids, 1, positions, 4096)
    where = {"payload": 32 + 777, "position": 8, "layer": 24, "request": 16, "version": 28, "digest": 1}
    bad = window.copy()
    for kind, rec in flips:
        bad[int(offsets[rec]) + where[kind]] ^= 0x10
    for g in (groups, None):
        want = ob.records_verify(bad, offsets, ids, request, 1, 4096, g)[:2]
        got = _gpu_verify(bad, offsets, ids, request, 1, 4096, g)[:2]
        assert want[0] in (90, 91) and got == want, (g is None, got, want)


def test_verify_bounds(cuda):
    img, payloads, request, positions = _store(4096)
    ids = np.arange(8, dtype=np.uint64)
    window, offsets, groups = _windows(img, ids, 0, positions, 4096)
    short = window[: int(offsets[5]) + 4096]  # record 5 truncated
    assert _gpu_verify(short, offsets, ids, request, 0, 4096)[:2] == (92, 5)
    assert _gpu_verify(window, offsets, ids, request, 0, 4096, out_rows=[0, 1, 2, 3, 4, 5, 6, 8])[:2] == (92, 7)


def test_full_size_encode_verify_round_trip(cuda):
    """Four layers x 32768 positions of 4096-byte K||V rows (512 MiB): the
    GPU encode of every record, verified back by the GPU, returns every
    payload; sampled records equal the oracle's images."""
    import torch
    import hillserve_b200 as hsb

    layers, positions, nbytes, request = 4, 32768, 4096, 4242
    g = torch.Generator(device="cuda").manual_seed(3)
    payload = torch.randint(0, 256, (layers * positions, nbytes), dtype=torch.uint8, device="cuda", generator=g)
    stride = nbytes + 32
    records = torch.empty(layers * positions * stride, dtype=torch.uint8, device="cuda")
    for l in range(layers):
        hsb.kv_records_encode(payload[l * positions:(l + 1) * positions], positions, nbytes, request, l, 0,
                              out=records[l * positions * stride:(l + 1) * positions * stride])
    out = torch.zeros_like(payload[:positions])
    for l in range(layers):
        offs = torch.arange(positions, dtype=torch.int64, device="cuda") * stride + l * positions * stride
        pos = torch.arange(positions, dtype=torch.int64, device="cuda")
        hsb.kv_records_verify(records, offs, pos, request, l, nbytes, out)
        assert torch.equal(out, payload[l * positions:(l + 1) * positions])
    sample = np.random.default_rng(0).choice(layers * positions, 64, replace=False)
    host = payload[torch.from_numpy(sample).cuda()].cpu().numpy()
    recs = records.view(-1, stride)[torch.from_numpy(sample).cuda()].cpu().numpy()
    for j, r in enumerate(sample):
        l, p = divmod(int(r), positions)
        assert np.array_equal(recs[j], ob.records_encode(host[j], 1, nbytes, request, l, p))


def test_verify_in_place_from_pinned_host_window(cuda):
    """The verifier reads the records straight from pinned host read buffers;
    pageable host memory is refused before any launch."""
    import torch
    import hillserve_b200 as hsb

    img, payloads, request, positions = _store(4096)
    ids = np.sort(np.random.default_rng(5).choice(positions, 61, replace=False)).astype(np.uint64)
    window, offsets, groups = _windows(img, ids, 1, positions, 4096)
    host = torch.from_numpy(window).pin_memory()
    out = torch.zeros((len(ids), 4096), dtype=torch.uint8, device="cuda")
    hsb.kv_records_verify(host, _dev(offsets.astype(np.int64)), _dev(ids.astype(np.int64)), request, 1, 4096, out,
                          groups=_dev(groups.astype(np.int32)))
    assert np.array_equal(out.cpu().numpy(), payloads[1][ids.astype(np.int64)])
    bad = window.copy()
    bad[int(offsets[17]) + 32 + 9] ^= 1
    st = hsb.kv_records_verify(torch.from_numpy(bad).pin_memory(), _dev(offsets.astype(np.int64)),
                               _dev(ids.astype(np.int64)), request, 1, 4096, out, check=False)
    torch.cuda.synchronize()
    assert st.cpu().numpy().tolist() == [91, 17]
    with pytest.raises(hsb.HsbError):
        hsb.kv_records_verify(torch.from_numpy(window), _dev(offsets.astype(np.int64)), _dev(ids.astype(np.int64)),
                              request, 1, 4096, out)
