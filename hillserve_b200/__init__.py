"""B200-native selected-KV decode path of HillServe.

Python mirror of the reference interfaces, over the C ABI of ``include/hsb.h``
(``libhsb.so``, hand-written sm_100a kernels).  PyTorch only supplies device
memory and streams; every computation runs in the CUDA library.

Reference interfaces mirrored here (paths inside the HillServe project):
  FullGqaCpuScorer            policy/full_gqa_cpu.hpp:27-50      -> FullGqaScorer
  select_gqa_scores           policy/gqa_policy.hpp:19-21        -> select_gqa_scores
  runtime score scaling       policy/full_gqa_runtime.cpp:571    -> scale_scores
  prefetch cover              policy/full_gqa_runtime.cpp:299-344 -> prefetch_cover
  gqa_physical_union          runtime/gqa_pack.hpp:12-22         -> gqa_physical_union
  pack_gqa_workspace          runtime/gqa_pack.hpp:26-58         -> pack_gqa_workspace
  GQAPrefetchCuda             runtime/gqa_prefetch_cuda.hpp:8-25 -> GQAPrefetchCuda
  GQADeliveryWorkspace        runtime/gqa_delivery.hpp:10-19     -> GQADeliveryWorkspace
  rehearsal query (ggml)      patches/llama-b6000-round2.patch:303-317 -> rehearsal_query

Errors: the reference throws std::invalid_argument for scorer / union / pack
shape errors and std::runtime_error for selector and delivery errors; here
they raise ``InvalidArgument`` (a ValueError) and ``HsbError`` (a
RuntimeError) with the same messages.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

from ._capi import DeviceStatus, HsbError, KeyView, LayerBuffers, Selection, lib

__all__ = [
    "HsbError", "InvalidArgument", "FullGqaScorer", "score_full_gqa", "score_pipeline_v3",
    "scale_scores", "GQASelection", "select_gqa_scores", "prefetch_cover", "gqa_physical_union",
    "pack_gqa_workspace", "gather_map", "gather_cache", "stage_rows", "attention_packed",
    "attention_dense", "rehearsal_query", "GQAPrefetchCuda", "GQADeliveryWorkspace",
    "SelectedKVLayer", "attention_slots", "h2o_group_sums", "GQAH2OStatsCuda",
    "segment_header", "segment_extent_bytes", "kv_records_encode", "kv_records_verify", "kv_read_plan",
    "kv_read_groups", "plan_hot_slots", "score_history", "History", "DecodeExecutor",
]

# Status codes the reference reports as std::invalid_argument.
_INVALID_ARGUMENT = {10, 11, 12, 30, 31, 40, 41, 42, 43, 93}


class InvalidArgument(HsbError, ValueError):
    """Stands for the reference's std::invalid_argument."""


def _raise(status: int) -> None:
    if status == 0:
        return
    msg = lib().hsb_last_error().decode() or lib().hsb_status_message(status).decode()
    if status in _INVALID_ARGUMENT:
        raise InvalidArgument(status, msg)
    raise HsbError(status, msg)


def _torch():
    import torch
    return torch


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t) -> C.c_void_p:
    """The address a kernel will read or write.  Device tensors and pinned
    host tensors (mapped into the GPU's address space) qualify; a pageable
    host tensor would make the kernel fault, so it is refused here."""
    if t is None:
        return C.c_void_p(0)
    if t.device.type == "cpu" and not t.is_pinned():
        raise InvalidArgument(10, "a pageable host tensor cannot be read by the GPU: pass a device or pinned tensor")
    return C.c_void_p(t.data_ptr())


def _status_buffer(device):
    torch = _torch()
    return torch.zeros(2, dtype=torch.int32, device=device)


def _check_status(st, stream=None) -> None:
    _raise(lib().hsb_status_check(_ptr(st), _stream(stream)))


def _workspace(nbytes: int, device):
    torch = _torch()
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def _u16(t):
    torch = _torch()
    if t.dtype in (torch.float16, torch.int16, torch.bfloat16):
        return t
    if t.dtype == torch.uint16:
        return t.view(torch.int16)
    raise TypeError(f"expected a 16-bit tensor, got {t.dtype}")


# ---------------------------------------------------------------- stage 1
def _views(views) -> tuple:
    arr = (KeyView * max(1, len(views)))()
    total = 0
    for i, v in enumerate(views):
        data, tokens, stride = v
        arr[i] = KeyView(data.data_ptr() if hasattr(data, "data_ptr") else int(data), int(tokens), int(stride))
        total += int(tokens)
    return arr, total


def score_full_gqa(query, views: Sequence, out=None, stream=None):
    """Scores F16 query [32*128] against concatenated key views.

    ``views`` is a sequence of (tensor, tokens, stride_words) with stride 1024
    (token-major K) or 2048 (interleaved K|V rows).  Returns int16 bits of the
    F16 scores, shape [32, sum tokens], head-major (full_gqa_cpu.cpp:206-250).
    """
    torch = _torch()
    arr, total = _views(views)
    if out is None:
        out = torch.empty((32, max(total, 1)), dtype=torch.int16, device=query.device)
    _raise(lib().hsb_score_views(_ptr(query), arr, len(views), _ptr(out), _stream(stream)))
    return out


def score_pipeline_v3(query, keys, tokens: int, out=None, stream=None):
    """The V3 pipeline contract: 64 <= tokens <= 32768, tokens % 64 == 0."""
    torch = _torch()
    if out is None:
        out = torch.empty((32, max(int(tokens), 1)), dtype=torch.int16, device=query.device)
    _raise(lib().hsb_score_pipeline_v3(_ptr(query), _ptr(keys), C.c_uint32(int(tokens) & 0xffffffff), _ptr(out),
                                        _stream(stream)))
    return out


class FullGqaScorer:
    """Mirror of FullGqaCpuScorer (policy/full_gqa_cpu.hpp:27-50) on the GPU.

    ``threads``/``implementation`` are validated as the reference does (1..128;
    automatic/scalar/avx2_f16c) so existing configurations keep working; they
    do not change the kernel, which is always the sm_100a scorer.
    """

    IMPLEMENTATIONS = ("automatic", "scalar", "avx2_f16c")

    def __init__(self, threads: int = 1, implementation: str = "automatic"):
        if threads == 0 or threads > 128:
            raise InvalidArgument(10, "full GQA CPU threads must be 1..128")
        if implementation not in self.IMPLEMENTATIONS:
            raise InvalidArgument(10, "unknown full GQA CPU implementation")
        self._threads = threads

    def threads(self) -> int:
        return self._threads

    def implementation_name(self) -> str:
        return "sm100a_ordered_fp32"

    def score(self, query, views: Sequence, output=None, stream=None):
        if output is not None and output.data_ptr() == query.data_ptr():
            raise InvalidArgument(11, "full GQA CPU output must not alias the query")
        if query.numel() != 32 * 128 or len(views) == 0:
            raise InvalidArgument(10, "full GQA CPU query/views shape")
        return score_full_gqa(query, views, output, stream)


def scale_scores(raw, out=None, stream=None):
    """F16(F32(raw) / sqrtf(128)) elementwise (full_gqa_runtime.cpp:571)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(raw)
    _raise(lib().hsb_scale_scores(_ptr(raw), raw.numel(), _ptr(out), _stream(stream)))
    return out


# ---------------------------------------------------------------- stage 2
@dataclass
class GQASelection:
    """Mirror of GQASelection (policy/gqa_policy.hpp:14-18).  ``ids`` is an
    int32 device tensor [heads, k] (rows are the ordered per-head lists)."""
    ids: object
    counts: list
    k: int
    boundary_tied_heads: int
    ids_buffer: object = field(default=None, repr=False)


def select_kmax(valid: int, ratio: float) -> int:
    return min(int(math.floor(float(valid) * float(C.c_float(ratio).value))), int(valid))


def select_gqa_scores(scores, heads: int, stride: int, valid_tokens: int, alpha: float, cap_ratio: float,
                      fp32_counts: bool = False, *, raw: bool = False, stream=None) -> GQASelection:
    """select_gqa_scores (gqa_policy.cpp:47-70), synchronous like the reference.

    With ``raw=True`` the scores are raw dot products and are normalised in
    the kernel (the runtime's scale-then-select, full_gqa_runtime.cpp:571-572).
    """
    torch = _torch()
    dev = scores.device
    kcap = max(1, select_kmax(valid_tokens, cap_ratio)) if 0 < valid_tokens <= stride else 1
    ids = torch.empty((max(1, heads), kcap), dtype=torch.int32, device=dev)
    counts = torch.zeros(max(1, heads), dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int32, device=dev)
    ws = _workspace(lib().hsb_select_workspace_bytes(heads, stride, valid_tokens, kcap), dev)
    _raise(lib().hsb_select(_ptr(scores), int(raw), heads, stride, valid_tokens, C.c_float(alpha),
                            C.c_float(cap_ratio), int(fp32_counts), _ptr(ids), kcap, _ptr(counts), _ptr(result),
                            _ptr(ws), ws.numel(), _stream(stream)))
    host = Selection()
    _raise(lib().hsb_selection_read(_ptr(result), C.byref(host), _stream(stream)))
    k = int(host.k)
    return GQASelection(ids=ids[:, :k], counts=[int(c) & 0xffffffff for c in counts.cpu().tolist()], k=k,
                        boundary_tied_heads=int(host.boundary_tied_heads), ids_buffer=ids)


def prefetch_cover(raw, capacity: int, position: int, alpha: float, fp32_counts: bool = False, stream=None):
    """History-only prefetch cover (full_gqa_runtime.cpp:299-344).

    ``raw``: raw F16 scores [32, capacity].  Returns (per_head int32 [32, bound],
    physical int32 sorted union)."""
    torch = _torch()
    dev = raw.device
    cap = min(int(position), int(math.floor(float(position + 1) * float(C.c_float(0.2).value))))
    per_head = torch.empty((32, max(cap, 1)), dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int32, device=dev)
    ws = _workspace(lib().hsb_select_workspace_bytes(32, capacity, max(position, 1), max(cap, 1)), dev)
    _raise(lib().hsb_prefetch_cover(_ptr(raw), capacity, position, C.c_float(alpha), int(fp32_counts), _ptr(per_head),
                                    cap, _ptr(result), _ptr(ws), ws.numel(), _stream(stream)))
    host = Selection()
    _raise(lib().hsb_selection_read(_ptr(result), C.byref(host), _stream(stream)))
    bound = int(host.k)
    sizes = torch.full((32,), bound, dtype=torch.int32, device=dev)
    physical = gqa_physical_union(per_head, sizes, position, stream=stream)
    return per_head[:, :bound], physical


# ---------------------------------------------------------------- stage 3
def gqa_physical_union(ids, sizes, visible: int, stream=None):
    """gqa_physical_union (gqa_pack.hpp:12-22).  ``ids`` int32 [32, kstride],
    ``sizes`` int32 [32] device tensor.  Returns the sorted int32 union."""
    torch = _torch()
    dev = ids.device
    kstride = ids.shape[1] if ids.dim() == 2 else 0
    physical = torch.empty(max(1, int(visible)), dtype=torch.int32, device=dev)
    count = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _status_buffer(dev)
    ws = _workspace(lib().hsb_union_workspace_bytes(max(1, int(visible))), dev)
    _raise(lib().hsb_union(_ptr(ids), kstride, _ptr(sizes), 1, int(visible), _ptr(physical), _ptr(count), _ptr(st),
                           _ptr(ws), ws.numel(), _stream(stream)))
    _check_status(st, stream)
    return physical[: int(count.item())]


def pack_gqa_workspace(ids, sizes, positions, physical, payload, count: int, k, v, mask=None, stream=None):
    """pack_gqa_workspace (gqa_pack.hpp:26-58) into device tensors k, v
    (int16 [count*4096]) and mask (float32 [32*qpad*count]), synchronous."""
    torch = _torch()
    dev = k.device
    pos = positions if torch.is_tensor(positions) else torch.tensor(list(positions), dtype=torch.int64, device=dev)
    npos = pos.numel()
    last = int(pos[-1].item()) if npos else 0
    nphys = physical.numel()
    st = _status_buffer(dev)
    ws = _workspace(lib().hsb_pack_workspace_bytes(min(last, 66047)), dev)
    kstride = ids.shape[1] if ids.dim() == 2 else 0
    _raise(lib().hsb_pack(_ptr(ids), kstride, _ptr(sizes), 1, _ptr(pos), npos, last, _ptr(physical), nphys,
                          _ptr(payload), payload.numel() * payload.element_size(), int(count), _ptr(k), _ptr(v),
                          _ptr(mask), _ptr(st), _ptr(ws), ws.numel(), _stream(stream)))
    _check_status(st, stream)


def gather_map(prefetched, prefetched_rows: int, misses, miss_rows: int, row_map, count: int, k, v, stream=None):
    """gather_gqa (gqa_prefetch_cuda.cu:12-22) with deliver's row checks."""
    st = _status_buffer(k.device)
    _raise(lib().hsb_gather_map(_ptr(prefetched), prefetched_rows, _ptr(misses), miss_rows, _ptr(row_map), int(count),
                                _ptr(k), _ptr(v), _ptr(st), _stream(stream)))
    _check_status(st, stream)


def gather_cache(ids, sizes, sizes_stride: int, kcache, vcache, stride_words: int, visible: int, count: int, k, v,
                 zero_padding: bool = True, status=None, stream=None):
    """Device-resident gather of selected rows from an HBM KV cache."""
    kstride = ids.shape[1] if ids.dim() == 2 else int(count)
    _raise(lib().hsb_gather_cache(_ptr(ids), kstride, _ptr(sizes), sizes_stride, _ptr(kcache), _ptr(vcache),
                                  stride_words, visible, count, int(zero_padding), _ptr(k), _ptr(v), _ptr(status),
                                  _stream(stream)))


def stage_rows(rows, physical, count, max_rows: int, dst, stream=None):
    """dst[i] = rows[physical[i]] (4096-byte rows) for i < count; rows may be
    mapped pinned host memory (the cold tier)."""
    ptr = rows if isinstance(rows, int) else rows.data_ptr()
    _raise(lib().hsb_stage_rows(C.c_void_p(ptr), _ptr(physical), _ptr(count), max_rows, _ptr(dst), _stream(stream)))


# ---------------------------------------------------------------- stage 4
def attention_packed(q, k, v, count: int, mask=None, qpad: int = 0, sizes=None, sizes_stride: int = 1, out=None,
                     stream=None):
    """softmax(K.q/sqrt(128) + mask).V per query head over the packed layout."""
    torch = _torch()
    dev = q.device
    if out is None:
        out = torch.empty((32, 128), dtype=torch.float32, device=dev)
    ws = _workspace(lib().hsb_attention_workspace_bytes(int(count)), dev)
    _raise(lib().hsb_attention_packed(_ptr(q), _ptr(k), _ptr(v), int(count), _ptr(mask), int(qpad), _ptr(sizes),
                                      sizes_stride, _ptr(out), _ptr(ws), ws.numel(), _stream(stream)))
    return out


def attention_dense(q, kcache, vcache, tokens: int, stride_words: int, out=None, stream=None):
    torch = _torch()
    dev = q.device
    if out is None:
        out = torch.empty((32, 128), dtype=torch.float32, device=dev)
    ws = _workspace(lib().hsb_attention_dense_workspace_bytes(int(tokens)), dev)
    _raise(lib().hsb_attention_dense(_ptr(q), _ptr(kcache), _ptr(vcache), int(tokens), int(stride_words), _ptr(out),
                                     _ptr(ws), ws.numel(), _stream(stream)))
    return out


# ------------------------------------------------------------ rehearsal
def rehearsal_query(x, w, position: int, theta: float = 500000.0, stream=None):
    """q = RoPE_position(W x): returns (F32 [32,128], F16 bits int16 [32,128])."""
    torch = _torch()
    dev = x.device
    q32 = torch.empty((32, 128), dtype=torch.float32, device=dev)
    q16 = torch.empty((32, 128), dtype=torch.int16, device=dev)
    _raise(lib().hsb_rehearsal_query(_ptr(x), _ptr(w), int(position), C.c_float(theta), _ptr(q32), _ptr(q16),
                                     _stream(stream)))
    return q32, q16


# ---------------------------------------------------- synthetic inputs
def synth_normal(count: int, seed: int, stddev: float = 1.0, bf16: bool = False, out=None, device="cuda",
                 stream=None):
    """Seeded N(0, stddev) values as F16 (or BF16) bits, int16 [count]
    (hsb_synth_normal_f16 / _bf16; reproducible on the CPU bit for bit)."""
    torch = _torch()
    if out is None:
        out = torch.empty(int(count), dtype=torch.int16, device=device)
    fn = lib().hsb_synth_normal_bf16 if bf16 else lib().hsb_synth_normal_f16
    _raise(fn(_ptr(out), int(count), int(seed), C.c_float(stddev), _stream(stream)))
    return out


def synth_keys(tokens: int, seed: int, heavy_fraction: float = 0.02, heavy_scale: float = 4.0, rope: bool = True,
               theta: float = 500000.0, stride_words: int = 1024, out=None, device="cuda", stream=None):
    """Seeded key rows [tokens][stride_words] (1024 words written per row):
    N(0,1) F16 values, a heavy_fraction of rows times heavy_scale, NORM-mode
    RoPE by token position (hsb_synth_keys)."""
    torch = _torch()
    if out is None:
        out = torch.empty(int(tokens) * int(stride_words), dtype=torch.int16, device=device)
    _raise(lib().hsb_synth_keys(_ptr(out), int(tokens), int(stride_words), int(seed), C.c_float(heavy_fraction),
                                C.c_float(heavy_scale), int(rope), C.c_float(theta), _stream(stream)))
    return out


def attention_slots(position: int, ratio: float = 0.2) -> int:
    """Reference delivery slot count max(32, roundup32(floor(0.2*(pos+1))))
    (runtime/gqa_executor.cpp:145)."""
    return max(32, (int(math.floor((position + 1) * ratio)) + 31) // 32 * 32)


# ------------------------------------------------------- H2O statistics
def _h2o_args(ne, nb):
    ne_arr = (C.c_int64 * 4)(*[int(x) for x in ne])
    nb_arr = (C.c_size_t * 4)(*[int(x) for x in nb])
    return ne_arr, nb_arr


def h2o_group_sums(probabilities, ne, byte_strides, valid_keys: int, valid_queries: int, out=None,
                   stream=None):
    """Device-resident H2O group sums (runtime/gqa_h2o_stats.cu:41-57):
    F32 [8, valid_keys] on the probabilities' device, enqueued on `stream`.
    `probabilities` is a CUDA tensor (its storage holds the F32 softmax with
    ggml byte strides) or a raw device address (int)."""
    torch = _torch()
    dev = probabilities.device if hasattr(probabilities, "device") else torch.device("cuda")
    if out is None:
        out = torch.empty((8, max(int(valid_keys), 1)), dtype=torch.float32, device=dev)
    ptr = C.c_void_p(probabilities.data_ptr() if hasattr(probabilities, "data_ptr") else int(probabilities))
    ne_arr, nb_arr = _h2o_args(ne, byte_strides)
    cap = out.numel() // 8
    _raise(lib().hsb_h2o_group_sums(ptr, ne_arr, nb_arr, int(valid_keys), int(valid_queries), _ptr(out), cap, None,
                                    _stream(stream)))
    return out


@dataclass
class H2OResult:
    """GQAH2OStatsCuda::Result (runtime/gqa_h2o_stats.hpp:16-25); `sums` is
    [8 * valid_keys] F32 in pinned host memory, borrowed until the next
    reduce()."""
    sums: object = None
    elements: int = 0
    started_ns: int = 0
    ready_observed_ns: int = 0
    d2h_bytes: int = 0
    reduction_ms: float = 0.0
    d2h_ms: float = 0.0


class GQAH2OStatsCuda:
    """runtime/gqa_h2o_stats.hpp:12-45 on B200: 8 x capacity_keys F32 on the
    device and in pinned host memory; reduce() runs the group-sum kernel on
    the caller's attention stream, copies the sums to the host and waits for
    them, timing both with events."""

    def __init__(self, actual_gpu_tensor, capacity_keys: int):
        torch = _torch()
        if actual_gpu_tensor is None or not capacity_keys:
            raise HsbError(80, "H2O statistics needs CUDA pointer and nonzero capacity")
        if not getattr(actual_gpu_tensor, "is_cuda", False):
            raise HsbError(80, "H2O attention statistics requires CUDA device memory")
        self.device = actual_gpu_tensor.device
        self.capacity = int(capacity_keys)
        self._gpu = torch.empty(8 * self.capacity, dtype=torch.float32, device=self.device)
        self._host = torch.empty(8 * self.capacity, dtype=torch.float32, pin_memory=True)
        self._events = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def gpu_bytes(self) -> int:
        return 8 * self.capacity * 4

    def host_bytes(self) -> int:
        return 8 * self.capacity * 4

    def reduce(self, probabilities, ne, byte_strides, valid_keys: int, valid_queries: int, stream) -> H2OResult:
        import time

        torch = _torch()
        if stream is None:
            raise HsbError(80, "H2O reduction invalid pointer, actual CUDA stream or capacity")
        if probabilities.device != self.device:
            raise HsbError(80, "H2O softmax tensor is not on the expected CUDA device")
        keys = int(valid_keys)
        out = H2OResult(elements=8 * keys, d2h_bytes=8 * keys * 4, started_ns=time.monotonic_ns())
        begin, reduced, copied = self._events
        ptr = C.c_void_p(probabilities.data_ptr())
        ne_arr, nb_arr = _h2o_args(ne, byte_strides)
        with torch.cuda.stream(stream):
            begin.record(stream)
            _raise(lib().hsb_h2o_group_sums(ptr, ne_arr, nb_arr, keys, int(valid_queries), _ptr(self._gpu),
                                            self.capacity, None, _stream(stream)))
            reduced.record(stream)
            self._host[:8 * keys].copy_(self._gpu[:8 * keys], non_blocking=True)
            copied.record(stream)
        copied.synchronize()
        out.ready_observed_ns = time.monotonic_ns()
        out.reduction_ms = begin.elapsed_time(reduced)
        out.d2h_ms = reduced.elapsed_time(copied)
        out.sums = self._host[:8 * keys].numpy()
        return out


# ------------------------------------------------- cold-tier KV records
def segment_extent_bytes(layers: int, positions: int, record_bytes: int) -> int:
    """Page-rounded SegmentedKVStore v1 file extent (segmented_store.cpp:26)."""
    n = lib().hsb_segment_extent_bytes(int(layers), int(positions), int(record_bytes))
    if not n:
        raise HsbError(93, "bounded segmented geometry/quota")
    return int(n)


def segment_header(request: int, layers: int, positions: int, record_bytes: int) -> bytes:
    """The 4096-byte file header (segmented_store.cpp:30)."""
    buf = C.create_string_buffer(4096)
    _raise(lib().hsb_segment_header(buf, int(request), int(layers), int(positions), int(record_bytes)))
    return buf.raw


def kv_records_encode(payload, count: int, record_bytes: int, request: int, layer: int, first: int,
                      payload_stride: Optional[int] = None, out=None, stream=None):
    """File image of records (layer, first + i), i < count, from device
    payload rows: uint8 [count * (record_bytes + 32)] on the payload's device."""
    torch = _torch()
    if out is None:
        out = torch.empty(int(count) * (int(record_bytes) + 32), dtype=torch.uint8, device=payload.device)
    stride = int(record_bytes) if payload_stride is None else int(payload_stride)
    _raise(lib().hsb_kv_records_encode(_ptr(payload), stride, int(count), int(record_bytes), int(request),
                                       int(layer), int(first), _ptr(out), _stream(stream)))
    return out


def kv_records_verify(window, offsets, positions, request: int, layer: int, record_bytes: int, out,
                      groups=None, out_rows=None, check: bool = True, stream=None):
    """Checks records of a window (device memory, or pinned host memory read
    in place) and gathers their payloads into the device rows `out`.  offsets / positions: uint64 (int64)
    device tensors; groups, out_rows: optional int32 device tensors.
    Raises the reference's error (check=True) or returns the status tensor."""
    st = _status_buffer(out.device)
    count = int(offsets.numel())
    stride = out.stride(0) * out.element_size() if out.dim() > 1 else int(record_bytes)
    capacity = out.numel() * out.element_size() // stride
    _raise(lib().hsb_kv_records_verify(_ptr(window), window.numel() * window.element_size(), _ptr(offsets),
                                       _ptr(positions), _ptr(groups), count, int(request), int(layer),
                                       int(record_bytes), _ptr(out), stride, _ptr(out_rows), capacity, _ptr(st),
                                       _stream(stream)))
    if check:
        _check_status(st, stream)
    return st


class KVReadWindow(C.Structure):
    _fields_ = [("begin", C.c_uint64), ("end", C.c_uint64), ("required_page_bytes", C.c_uint64),
                ("first_record", C.c_uint64), ("end_record", C.c_uint64)]


def kv_read_plan(offsets, record_bytes: int, extent: int, window_bytes: int = 1 << 20, gap_bytes: int = 16 << 10,
                 max_amplification_permille: int = 1500) -> list:
    """storage/kv_read_plan.hpp:34-59 on the host: [(begin, end,
    required_page_bytes, first_record, end_record), ...]."""
    offs = [int(o) for o in offsets]
    arr = (C.c_uint64 * max(1, len(offs)))(*offs)
    wins = (KVReadWindow * max(1, len(offs)))()
    n = C.c_size_t(0)
    _raise(lib().hsb_kv_read_plan(arr, len(offs), int(record_bytes), int(extent), int(window_bytes), int(gap_bytes),
                                  int(max_amplification_permille), wins, len(wins), C.byref(n)))
    return [(w.begin, w.end, w.required_page_bytes, w.first_record, w.end_record) for w in wins[:n.value]]


def kv_read_groups(windows: list, count: int) -> list:
    """The reference's validation groups (batches of four per window)."""
    wins = (KVReadWindow * max(1, len(windows)))(*[KVReadWindow(*w) for w in windows])
    out = (C.c_uint32 * max(1, count))()
    _raise(lib().hsb_kv_read_groups(wins, len(windows), out, int(count)))
    return list(out[:count])


# ------------------------------------------------------- decode history
class HistoryConfig(C.Structure):
    _fields_ = [("layers", C.c_size_t), ("capacity", C.c_size_t), ("prompt_tokens", C.c_size_t),
                ("generated_capacity", C.c_size_t), ("alpha", C.c_float), ("fp32_counts", C.c_int)]


def plan_hot_slots(prompt_tokens: int, generated_capacity: int, capacity: int, beta: float = 1.0,
                   allow_partial_prompt: bool = False):
    """plan_full_gqa_runtime's placement (runtime/full_gqa_contract.hpp):
    (hot_slot_by_position int64 [capacity], prompt hot tokens)."""
    import numpy as np

    out = np.zeros(int(capacity), dtype=np.int64)
    hot = C.c_size_t(0)
    _raise(lib().hsb_history_plan_slots(int(prompt_tokens), int(generated_capacity), int(capacity), float(beta),
                                        int(allow_partial_prompt), out.ctypes.data, C.byref(hot)))
    return out, hot.value


def score_history(q, hot_pool, cold_k, row_of_position, valid: int, out=None, order_keys=None, stream=None):
    """Raw V3 scores of positions [0, valid) whose K rows live in a hot pool
    (rows of 2048 words) or a cold K store (rows of 1024 words); see
    hsb_score_history.  row_of_position: host int64 array."""
    import numpy as np

    torch = _torch()
    rows = np.ascontiguousarray(row_of_position, dtype=np.int64)
    if out is None:
        out = torch.empty((32, int(valid)), dtype=torch.int16, device=q.device)
    stride = out.stride(0)
    _raise(lib().hsb_score_history(_ptr(_u16(q)), _ptr(hot_pool), 2048, _ptr(cold_k), 1024, rows.ctypes.data,
                                   int(valid), _ptr(out), stride, _ptr(order_keys), _stream(stream)))
    return out


class History:
    """FullGqaRuntimePolicy's decode history (policy/full_gqa_runtime.hpp:
    14-106) on the GPU: append / prepare_history / select / fetch of one
    request, the hot KV rows and every K row in HBM (hsb_history_*)."""

    def __init__(self, layers: int, capacity: int, prompt_tokens: int, generated_capacity: int, beta: float = 1.0,
                 alpha: float = 5.0, fp32_counts: bool = False, allow_partial_prompt: bool = False,
                 hot_slot_by_position=None):
        import numpy as np

        if hot_slot_by_position is None:
            hot_slot_by_position, _ = plan_hot_slots(prompt_tokens, generated_capacity, capacity, beta,
                                                     allow_partial_prompt)
        self.slots = np.ascontiguousarray(hot_slot_by_position, dtype=np.int64)
        cfg = HistoryConfig(layers, capacity, prompt_tokens, generated_capacity, alpha, int(fp32_counts))
        self.capacity = capacity
        self._h = C.c_void_p()
        _raise(lib().hsb_history_create(C.byref(cfg), self.slots.ctypes.data, C.byref(self._h)))
        self.kcap = lib().hsb_history_select_capacity(self._h)
        self.hot_slots = lib().hsb_history_hot_slots(self._h)
        self.cold_rows = lib().hsb_history_cold_rows(self._h)

    def close(self):
        if self._h:
            lib().hsb_history_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        self.close()

    def append(self, layer: int, first: int, rows, stream=None):
        """rows: [count][2048] 16-bit device tensor of K||V rows."""
        _raise(lib().hsb_history_append(self._h, layer, first, rows.shape[0], _ptr(_u16(rows)), _stream(stream)))

    def prepare_history(self, layer: int, position: int, q16, stream=None):
        _raise(lib().hsb_history_prepare(self._h, layer, position, _ptr(_u16(q16)), _stream(stream)))

    def cover(self, layer: int, stream=None):
        """(cold positions of the cover, ascending int32 device tensor; bound)."""
        torch = _torch()
        dev = torch.device("cuda")
        ids = torch.empty(self.capacity, dtype=torch.int32, device=dev)
        n = torch.zeros(1, dtype=torch.int32, device=dev)
        res = torch.zeros(4, dtype=torch.int32, device=dev)
        _raise(lib().hsb_history_cover(self._h, layer, _ptr(ids), _ptr(n), _ptr(res), _stream(stream)))
        count = int(n.item())
        if int(res[2].item()):
            _raise(int(res[2].item()))
        return ids[:count], int(res[0].item())

    def select(self, layer: int, position: int, q16, stream=None):
        """(ids int32 [32][kcap], counts int32 [32], result int32 [4] =
        {k, tied heads, status code, status index}) on the device; the
        tensors are the history's own, valid until its next select()."""
        torch = _torch()
        if not hasattr(self, "_ids"):
            dev = torch.device("cuda")
            self._ids = torch.zeros((32, max(self.kcap, 1)), dtype=torch.int32, device=dev)
            self._counts = torch.zeros(32, dtype=torch.int32, device=dev)
            self._res = torch.zeros(4, dtype=torch.int32, device=dev)
        _raise(lib().hsb_history_select(self._h, layer, position, _ptr(_u16(q16)), _ptr(self._ids),
                                        self._ids.shape[1], _ptr(self._counts), _ptr(self._res), _stream(stream)))
        return self._ids, self._counts, self._res

    def fetch(self, layer: int, ids, result, staged_ids, staged_rows, count: int, stream=None, check: bool = True,
              zero_padding: bool = True):
        """Packed K [count][32][128] and V [32][128][count] (int16) of the
        selection; cold rows from staged_rows (rows of the ascending
        staged_ids).  zero_padding=False writes the live slots only.  The
        tensors are the history's own, valid until its next fetch()."""
        torch = _torch()
        dev = torch.device("cuda")
        if getattr(self, "_count", None) != count:
            self._k = torch.zeros((count, 32, 128), dtype=torch.int16, device=dev)
            self._v = torch.zeros((32, 128, count), dtype=torch.int16, device=dev)
            self._count = count
            self._st = torch.zeros(2, dtype=torch.int32, device=dev)
        self._st.zero_()
        n = 0 if staged_ids is None else int(staged_ids.numel())
        _raise(lib().hsb_history_fetch(self._h, layer, _ptr(ids), ids.shape[1], _ptr(result), _ptr(staged_ids), n,
                                       _ptr(None if staged_rows is None else _u16(staged_rows)), count,
                                       int(zero_padding), _ptr(self._k), _ptr(self._v), _ptr(self._st),
                                       _stream(stream)))
        if check:
            _check_status(self._st, stream)
        return self._k, self._v, self._st


# ------------------------------------------------------ layer executor
class DecodeExecutor:
    """The model-facing decode step of GQALayerExecutor
    (runtime/gqa_executor.cpp:149-249) on the GPU: one HBM cache per layer,
    the model's current K/V appended by hsb_executor_append, attention over
    the selected live slots (hsb_executor_decode_layer)."""

    def __init__(self, layers: int, capacity: int, alpha: float = 5.0, ratio: float = 0.2, dense_layers: int = 2,
                 device=None):
        torch = _torch()
        dev = torch.device("cuda") if device is None else device
        self.layers, self.capacity, self.alpha, self.ratio, self.dense = layers, capacity, alpha, ratio, dense_layers
        self.count = max(32, (int(math.floor(capacity * ratio)) + 31) // 32 * 32)
        self.cache = [torch.zeros((capacity, 2048), dtype=torch.int16, device=dev) for _ in range(layers)]
        self.completed = [0] * layers
        ws = lib().hsb_executor_workspace_bytes(capacity, self.count)
        self.ws = torch.empty(ws, dtype=torch.uint8, device=dev)
        self.scores = torch.empty((32, capacity), dtype=torch.int16, device=dev)
        self.ids = torch.empty((32, self.count), dtype=torch.int32, device=dev)
        self.counts = torch.empty(32, dtype=torch.int32, device=dev)
        self.result = torch.zeros(4, dtype=torch.int32, device=dev)
        self.k_packed = torch.empty((self.count, 32, 128), dtype=torch.int16, device=dev)
        self.v_packed = torch.empty((32, 128, self.count), dtype=torch.int16, device=dev)
        self.status = torch.zeros(2, dtype=torch.int32, device=dev)

    def _buffers(self):
        return LayerBuffers(self.scores.data_ptr(), self.ids.data_ptr(), self.counts.data_ptr(),
                            self.result.data_ptr(), self.k_packed.data_ptr(), self.v_packed.data_ptr(),
                            self.ws.data_ptr(), self.ws.numel())

    def append(self, layer: int, current, stream=None):
        """current: F16 [n_tokens][8][256] (K 128 | V 128 per KV head)."""
        n = current.shape[0]
        _raise(lib().hsb_executor_append(_ptr(_u16(current)), n, _ptr(self.cache[layer]), self.capacity,
                                         self.completed[layer], _ptr(self.status), _stream(stream)))
        self.completed[layer] += n

    def decode_layer(self, layer: int, current, rehearsal, q, out=None, stream=None):
        """Appends the current token and returns the attention output F32 [32][128]."""
        torch = _torch()
        if out is None:
            out = torch.empty((32, 128), dtype=torch.float32, device=q.device)
        b = self._buffers()
        pos = self.completed[layer]
        _raise(lib().hsb_executor_decode_layer(_ptr(_u16(current)), _ptr(rehearsal), _ptr(q),
                                               _ptr(self.cache[layer]), self.capacity, pos,
                                               int(layer < self.dense), C.c_float(self.alpha),
                                               C.c_float(self.ratio), self.count, C.byref(b), _ptr(out),
                                               _ptr(self.status), _stream(stream)))
        self.completed[layer] += 1
        return out


# ------------------------------------------------------------ delivery
class GQAPrefetchCuda:
    """Mirror of GQAPrefetchCuda (runtime/gqa_prefetch_cuda.hpp:8-25).

    Two pinned staging slots and device row buffers; ``stage`` uploads a
    prefetched payload on a private stream and waits for it; ``deliver``
    makes the consumer stream wait for that upload, uploads misses and the row
    map, and runs the sm_100a gather into caller-owned K/V."""

    def __init__(self, device, max_rows: int):
        torch = _torch()
        self.device = torch.device(device)
        self.rows = int(max_rows)
        nbytes = self.rows * 4096
        self._host = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self._gpu = [torch.empty(nbytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self._streams = [torch.cuda.Stream(device=self.device) for _ in range(2)]
        self._ready = [torch.cuda.Event() for _ in range(2)]
        self._valid = [0, 0]
        self._misses = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self._map = torch.empty(self.rows * 32, dtype=torch.int32, device=self.device)

    def gpu_bytes(self) -> int:
        return self.rows * 4096 * 3 + self.rows * 32 * 4

    def host_bytes(self) -> int:
        return self.rows * 4096 * 2

    def stage(self, slot: int, payload: bytes) -> int:
        torch = _torch()
        if slot >= 2 or len(payload) > self.rows * 4096 or len(payload) % 4096:
            raise HsbError(50, "prefetch CUDA slot geometry")
        n = len(payload)
        if n:
            self._host[slot][:n].copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
        with torch.cuda.stream(self._streams[slot]):
            if n:
                self._gpu[slot][:n].copy_(self._host[slot][:n], non_blocking=True)
            self._ready[slot].record(self._streams[slot])
        self._ready[slot].synchronize()
        self._valid[slot] = n // 4096
        return n

    def deliver(self, slot: int, row_map: Sequence[int], misses: bytes, count: int, k, v, stream=None):
        torch = _torch()
        if slot >= 2 or count > self.rows or len(row_map) != count * 32 or len(misses) > self.rows * 4096 or \
                len(misses) % 4096:
            raise HsbError(50, "prefetch CUDA delivery geometry/stream")
        nmiss = len(misses) // 4096
        for row in row_map:  # deliver's host-side checks (gqa_prefetch_cuda.cu:218)
            if row >= 0 and row >= self._valid[slot]:
                raise HsbError(51, "prefetch row outside uploaded payload")
            if row <= -2 and -2 - row >= nmiss:
                raise HsbError(52, "prefetch miss row outside payload")
        s = stream if stream is not None else torch.cuda.current_stream()
        s.wait_event(self._ready[slot])
        with torch.cuda.stream(s):
            if nmiss:
                self._misses[: len(misses)].copy_(
                    torch.frombuffer(bytearray(misses), dtype=torch.uint8).pin_memory(), non_blocking=True)
            self._map[: len(row_map)].copy_(torch.tensor(list(row_map), dtype=torch.int32).pin_memory(),
                                            non_blocking=True)
        gather_map(self._gpu[slot], self._valid[slot], self._misses, nmiss, self._map, count, k, v, stream=s)
        s.synchronize()


class GQADeliveryWorkspace:
    """Mirror of GQADeliveryWorkspace (runtime/gqa_delivery.hpp:10-19): owns
    the packed K/V/mask workspace and the attention kernel (no ggml)."""

    def __init__(self, count: int, actual_attention_query, device="cuda"):
        torch = _torch()
        if not (0 < count <= 6592 and count % 32 == 0 and len(actual_attention_query) == 4096):
            raise HsbError(1, "bounded real GQA delivery shape")
        self.count = count
        self.device = torch.device(device)
        self.q = torch.as_tensor(actual_attention_query, dtype=torch.float32).reshape(32, 128).to(self.device)
        self.k = torch.empty(count * 4096, dtype=torch.int16, device=self.device)
        self.v = torch.empty(count * 4096, dtype=torch.int16, device=self.device)
        self.mask = torch.empty(count * 64 * 32, dtype=torch.float32, device=self.device)

    def gpu_bytes(self) -> int:
        return self.count * 4096 * 4 + self.count * 64 * 32 * 4

    def deliver(self, ids, sizes, position: int, physical, payload):
        pack_gqa_workspace(ids, sizes, [position], physical, payload, self.count, self.k, self.v, self.mask)

    def consume(self):
        return attention_packed(self.q, self.k, self.v, self.count, mask=self.mask, qpad=64)


class SelectedKVLayer:
    """One selected-KV decode layer over an HBM-resident KV cache, on one
    stream with no host round trip (hsb_layer_step): score -> select ->
    gather -> attention.  Buffers are allocated once for ``valid`` tokens."""

    def __init__(self, valid: int, alpha: float, ratio: float = 0.2, device="cuda"):
        torch = _torch()
        self.valid, self.alpha, self.ratio = int(valid), float(alpha), float(ratio)
        # Slot capacity: the largest k, rounded up to 32 so V rows stay aligned.
        self.count = max(32, (select_kmax(self.valid, self.ratio) + 31) // 32 * 32)
        dev = torch.device(device)
        self.scores = torch.empty((32, self.valid), dtype=torch.int16, device=dev)
        self.ids = torch.empty((32, self.count), dtype=torch.int32, device=dev)
        self.counts = torch.empty(32, dtype=torch.int32, device=dev)
        self.result = torch.zeros(4, dtype=torch.int32, device=dev)
        self.k_packed = torch.empty(self.count * 4096, dtype=torch.int16, device=dev)
        self.v_packed = torch.empty(self.count * 4096, dtype=torch.int16, device=dev)
        self.workspace = _workspace(lib().hsb_layer_workspace_bytes(self.valid, self.count), dev)
        self.out = torch.zeros((32, 128), dtype=torch.float32, device=dev)
        self._buffers = LayerBuffers(self.scores.data_ptr(), self.ids.data_ptr(), self.counts.data_ptr(),
                                     self.result.data_ptr(), self.k_packed.data_ptr(), self.v_packed.data_ptr(),
                                     self.workspace.data_ptr(), self.workspace.numel())

    def __call__(self, q16, q32, kcache, vcache, stride_words: int = 1024, out=None, stream=None):
        out = self.out if out is None else out
        _raise(lib().hsb_layer_step(_ptr(q16), _ptr(q32), _ptr(kcache), _ptr(vcache), stride_words, self.valid,
                                    C.c_float(self.alpha), C.c_float(self.ratio), self.count, C.byref(self._buffers),
                                    _ptr(out), _stream(stream)))
        return out

    def prepare(self, q16, kcache, stride_words: int = 1024, stream=None):
        """The history half (hsb_layer_prepare): scores positions [0, valid - 1)."""
        _raise(lib().hsb_layer_prepare(_ptr(q16), _ptr(kcache), stride_words, self.valid, C.c_float(self.alpha),
                                       C.c_float(self.ratio), self.count, C.byref(self._buffers), _stream(stream)))

    def select(self, q16, q32, kcache, vcache, stride_words: int = 1024, out=None, stream=None):
        """The select half (hsb_layer_select): scores the current position
        valid - 1, then selects, gathers and attends."""
        out = self.out if out is None else out
        _raise(lib().hsb_layer_select(_ptr(q16), _ptr(q32), _ptr(kcache), _ptr(vcache), stride_words, self.valid,
                                      C.c_float(self.alpha), C.c_float(self.ratio), self.count,
                                      C.byref(self._buffers), _ptr(out), _stream(stream)))
        return out

    def selection(self, stream=None) -> Selection:
        host = Selection()
        lib().hsb_selection_read(_ptr(self.result), C.byref(host), _stream(stream))
        return host
