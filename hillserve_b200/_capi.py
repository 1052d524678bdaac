"""ctypes declarations of the C ABI in ``include/hsb.h``.

The shared library is loaded from ``hillserve_b200/_lib/libhsb.so`` (built
in-tree by ``hillserve_b200.build``).  There is no other implementation: if
the library is missing every call raises, so nothing can silently run on a
CPU path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libhsb.so"

P = C.c_void_p
SZ = C.c_size_t
U64 = C.c_uint64
I = C.c_int
F = C.c_float


class KeyView(C.Structure):
    _fields_ = [("data", P), ("tokens", SZ), ("stride_words", SZ)]


class DeviceStatus(C.Structure):
    _fields_ = [("code", C.c_int32), ("index", C.c_int32)]


class MailboxLayout(C.Structure):
    _fields_ = [("thr", SZ), ("records", SZ), ("outputs", SZ), ("results", SZ), ("status", SZ), ("bytes", SZ)]


class PeerGroup(C.Structure):
    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("mailbox", P * 8), ("batch", SZ),
                ("wait_limit_ns", C.c_uint64)]


class Selection(C.Structure):
    _fields_ = [("k", C.c_uint32), ("boundary_tied_heads", C.c_uint32), ("status", DeviceStatus)]


class LayerBuffers(C.Structure):
    _fields_ = [
        ("scores", P), ("ids", P), ("counts", P), ("result", P),
        ("k_packed", P), ("v_packed", P), ("workspace", P), ("workspace_bytes", SZ),
    ]


# name: (restype, argtypes)
_SIGNATURES = {
    "hsb_abi_version": (I, []),
    "hsb_last_error": (C.c_char_p, []),
    "hsb_status_message": (C.c_char_p, [I]),
    "hsb_status_check": (I, [P, P]),
    "hsb_score_v3": (I, [P, P, SZ, SZ, P, P]),
    "hsb_score_views": (I, [P, P, SZ, P, P]),
    "hsb_score_pipeline_v3": (I, [P, P, C.c_uint32, P, P]),
    "hsb_score_with_keys": (I, [P, P, SZ, SZ, P, P, P]),
    "hsb_select_keys": (I, [P, P, SZ, SZ, SZ, F, F, I, P, SZ, P, P, P, SZ, P]),
    "hsb_scale_scores": (I, [P, SZ, P, P]),
    "hsb_select_workspace_bytes": (SZ, [SZ, SZ, SZ, SZ]),
    "hsb_select": (I, [P, I, SZ, SZ, SZ, F, F, I, P, SZ, P, P, P, SZ, P]),
    "hsb_selection_read": (I, [P, P, P]),
    "hsb_prefetch_cover": (I, [P, SZ, SZ, F, I, P, SZ, P, P, SZ, P]),
    "hsb_union_workspace_bytes": (SZ, [SZ]),
    "hsb_union": (I, [P, SZ, P, SZ, SZ, P, P, P, P, SZ, P]),
    "hsb_pack_workspace_bytes": (SZ, [U64]),
    "hsb_pack": (I, [P, SZ, P, SZ, P, SZ, U64, P, SZ, P, SZ, SZ, P, P, P, P, P, SZ, P]),
    "hsb_gather_map": (I, [P, SZ, P, SZ, P, SZ, P, P, P, P]),
    "hsb_gather_cache": (I, [P, SZ, P, SZ, P, P, SZ, SZ, SZ, I, P, P, P, P]),
    "hsb_stage_rows": (I, [P, P, P, SZ, P, P]),
    "hsb_attention_workspace_bytes": (SZ, [SZ]),
    "hsb_attention_packed": (I, [P, P, P, SZ, P, SZ, P, SZ, P, P, SZ, P]),
    "hsb_attention_packed_noalloc": (I, [P, P, P, SZ, P, SZ, P, SZ, P, P]),
    "hsb_attention_dense_workspace_bytes": (SZ, [SZ]),
    "hsb_attention_dense": (I, [P, P, P, SZ, SZ, P, P, SZ, P]),
    "hsb_rehearsal_query": (I, [P, P, U64, F, P, P, P]),
    "hsb_layer_workspace_bytes": (SZ, [SZ, SZ]),
    "hsb_layer_step": (I, [P, P, P, P, SZ, SZ, F, F, SZ, P, P, P]),
    "hsb_layer_prepare": (I, [P, P, SZ, SZ, F, F, SZ, P, P]),
    "hsb_layer_select": (I, [P, P, P, P, SZ, SZ, F, F, SZ, P, P, P]),
    "hsb_shard_head0_words": (SZ, []),
    "hsb_shard_score": (I, [P, I, P, SZ, SZ, P, P, P, P]),
    "hsb_shard_threshold": (I, [P, SZ, F, P, P]),
    "hsb_shard_count": (I, [P, SZ, SZ, SZ, P, P, P]),
    "hsb_shard_select_workspace_bytes": (SZ, [I, SZ, SZ, SZ]),
    "hsb_shard_select": (I, [P, P, I, SZ, SZ, P, P, SZ, SZ, F, F, P, SZ, P, P, P, P, P, P, P, P, P, SZ, P]),
    "hsb_mailbox_bytes": (SZ, [SZ]),
    "hsb_mailbox_layout_of": (None, [SZ, P]),
    "hsb_mailbox_create": (I, [SZ, P, P]),
    "hsb_mailbox_destroy": (I, [P]),
    "hsb_mailbox_open": (I, [P, P]),
    "hsb_mailbox_close": (I, [P]),
    "hsb_exchange_threshold": (I, [P, F, P, P]),
    "hsb_shard_score_push": (I, [P, I, P, SZ, SZ, P, P, P, F, P, P]),
    "hsb_exchange_count": (I, [P, SZ, SZ, P, P]),
    "hsb_exchange_finish": (I, [P, P, SZ, P, P]),
    "hsb_h2o_group_sums": (I, [P, P, P, SZ, SZ, P, SZ, P, P]),
    "hsb_segment_extent_bytes": (U64, [SZ, U64, SZ]),
    "hsb_segment_header": (I, [P, U64, SZ, U64, SZ]),
    "hsb_fnv1a64": (U64, [P, SZ]),
    "hsb_kv_records_encode": (I, [P, SZ, SZ, SZ, U64, C.c_uint32, U64, P, P]),
    "hsb_kv_records_verify": (I, [P, SZ, P, P, P, SZ, U64, C.c_uint32, SZ, P, SZ, P, SZ, P, P]),
    "hsb_kv_read_plan": (I, [P, SZ, U64, U64, SZ, SZ, C.c_uint, P, SZ, P]),
    "hsb_kv_read_groups": (I, [P, SZ, P, SZ]),
    "hsb_score_history": (I, [P, P, SZ, P, SZ, P, SZ, P, SZ, P, P]),
    "hsb_history_plan_slots": (I, [SZ, SZ, SZ, C.c_double, I, P, P]),
    "hsb_history_create": (I, [P, P, P]),
    "hsb_history_destroy": (None, [P]),
    "hsb_history_hot_slots": (SZ, [P]),
    "hsb_history_cold_rows": (SZ, [P]),
    "hsb_history_select_capacity": (SZ, [P]),
    "hsb_history_append": (I, [P, SZ, U64, SZ, P, P]),
    "hsb_history_prepare": (I, [P, SZ, U64, P, P]),
    "hsb_history_cover": (I, [P, SZ, P, P, P, P]),
    "hsb_history_select": (I, [P, SZ, U64, P, P, SZ, P, P, P]),
    "hsb_history_fetch": (I, [P, SZ, P, SZ, P, P, SZ, P, SZ, I, P, P, P, P]),
    "hsb_executor_append": (I, [P, SZ, P, SZ, SZ, P, P]),
    "hsb_executor_query": (I, [P, P, P, P]),
    "hsb_executor_workspace_bytes": (SZ, [SZ, SZ]),
    "hsb_executor_decode_layer": (I, [P, P, P, P, SZ, SZ, I, F, F, SZ, P, P, P, P]),
    "hsb_synth_normal_f16": (I, [P, SZ, U64, F, P]),
    "hsb_synth_normal_bf16": (I, [P, SZ, U64, F, P]),
    "hsb_synth_keys": (I, [P, SZ, SZ, U64, F, F, I, F, P]),
}

_lib = None


def declared_symbols() -> list[str]:
    """Names of every entry point this binding declares (all of hsb.h)."""
    return list(_SIGNATURES)


def lib() -> C.CDLL:
    """Loads libhsb.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m hillserve_b200.build` "
                "(the selected-KV path has no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class HsbError(RuntimeError):
    """A non-zero hsb_status; ``str()`` is the reference-worded message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int) -> None:
    if status != 0:
        raise HsbError(status, lib().hsb_last_error().decode() or lib().hsb_status_message(status).decode())
