"""numpy front end of the C oracle and of the reference bridge (tests only).

Every function takes and returns numpy arrays; uint16 arrays hold F16 bits.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libhs_oracle.so"
REF_SO = HERE / "_ref" / "libhs_ref.so"
REF_RUNTIME_SO = HERE / "_ref" / "libhs_ref_runtime.so"

P = C.c_void_p
SZ = C.c_size_t

_oracle = None
_ref = None


def build(reference_root: str | None = None) -> None:
    """Builds the oracle (and the reference bridge when its sources exist)."""
    cmd = ["make", "-s", "-C", str(HERE)]
    if reference_root:
        cmd.append(f"R={reference_root}")
    subprocess.run(cmd, check=True)


def _p(a) -> C.c_void_p:
    return C.c_void_p(0 if a is None else a.ctypes.data)


def oracle() -> C.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            build()
        lib = C.CDLL(str(ORACLE_SO))
        lib.orc_half_value.restype = C.c_float
        lib.orc_half_value.argtypes = [C.c_uint16]
        lib.orc_half_bits.restype = C.c_uint16
        lib.orc_half_bits.argtypes = [C.c_float]
        lib.orc_order_key.restype = C.c_uint16
        lib.orc_order_key.argtypes = [C.c_uint16]
        lib.orc_score.argtypes = [P, P, SZ, SZ, P, SZ, SZ, C.c_int]
        lib.orc_scale.argtypes = [P, SZ, P]
        lib.orc_scale.restype = None
        lib.orc_select.argtypes = [P, SZ, SZ, SZ, C.c_float, C.c_float, C.c_int, P, SZ, P, P, P]
        lib.orc_union.argtypes = [P, SZ, P, SZ, P, P]
        lib.orc_pack.argtypes = [P, SZ, P, P, SZ, P, SZ, P, SZ, SZ, P, P, P]
        lib.orc_gather_map.argtypes = [P, SZ, P, SZ, P, SZ, P, P]
        lib.orc_prefetch_cover.argtypes = [P, SZ, SZ, C.c_float, C.c_int, P, P, P, P]
        lib.orc_attention_packed.argtypes = [P, P, P, SZ, SZ, P, P]
        lib.orc_attention_packed.restype = None
        lib.orc_attention_compact.argtypes = [P, P, SZ, P, P, P]
        lib.orc_attention_compact.restype = None
        lib.orc_attention_dense.argtypes = [P, P, SZ, SZ, P, P]
        lib.orc_attention_dense.restype = None
        lib.orc_attention_dense_f32.argtypes = [P, P, SZ, SZ, P, P, C.c_int]
        lib.orc_attention_dense_f32.restype = None
        lib.orc_attention_packed_f32.argtypes = [P, P, P, SZ, SZ, P, P, C.c_int]
        lib.orc_attention_packed_f32.restype = None
        lib.orc_rehearsal.argtypes = [P, P, C.c_uint64, C.c_double, P]
        lib.orc_rehearsal.restype = None
        lib.orc_h2o_group_sums.argtypes = [P, SZ, SZ, SZ, SZ, SZ, P]
        lib.orc_h2o_group_sums.restype = None
        lib.orc_fnv1a64.argtypes = [P, SZ]
        lib.orc_fnv1a64.restype = C.c_uint64
        lib.orc_kv_records_encode.argtypes = [P, SZ, SZ, SZ, C.c_uint64, C.c_uint32, C.c_uint64, P]
        lib.orc_kv_records_encode.restype = None
        lib.orc_kv_records_verify.argtypes = [P, SZ, P, P, P, SZ, C.c_uint64, C.c_uint32, SZ, P, SZ, P, SZ, P]
        lib.orc_synth_normal.argtypes = [P, SZ, C.c_uint64, C.c_float, C.c_int, C.c_int]
        lib.orc_synth_normal.restype = None
        lib.orc_synth_keys.argtypes = [P, SZ, SZ, C.c_uint64, C.c_float, C.c_float, C.c_int, C.c_float, C.c_int]
        lib.orc_synth_keys.restype = None
        _oracle = lib
    return _oracle


def reference_available() -> bool:
    return REF_SO.exists()


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        lib = C.CDLL(str(REF_SO))
        lib.ref_half_value.restype = C.c_float
        lib.ref_half_value.argtypes = [C.c_uint16]
        lib.ref_half_bits.restype = C.c_uint16
        lib.ref_half_bits.argtypes = [C.c_float]
        lib.ref_scorer_create.restype = P
        lib.ref_scorer_create.argtypes = [C.c_uint, C.c_int, C.c_char_p, SZ]
        lib.ref_scorer_destroy.argtypes = [P]
        lib.ref_scorer_name.restype = C.c_char_p
        lib.ref_scorer_name.argtypes = [P]
        lib.ref_scorer_score.argtypes = [P, P, P, P, P, SZ, P, SZ, C.c_char_p, SZ]
        lib.ref_legacy_score.argtypes = [P, P, SZ, SZ, C.c_uint, P, C.c_char_p, SZ]
        lib.ref_scale.argtypes = [P, SZ, P]
        lib.ref_scale.restype = None
        lib.ref_select.argtypes = [P, SZ, SZ, SZ, C.c_float, C.c_float, C.c_int, P, SZ, P, P, P, C.c_char_p, SZ]
        lib.ref_union.argtypes = [P, SZ, P, SZ, P, P, C.c_char_p, SZ]
        lib.ref_pack.argtypes = [P, SZ, P, P, SZ, P, SZ, P, SZ, SZ, P, P, P, C.c_char_p, SZ]
        lib.ref_h2o_create.restype = P
        lib.ref_h2o_create.argtypes = [SZ, SZ, SZ, SZ, SZ, SZ, C.c_uint64, C.c_char_p, SZ]
        lib.ref_h2o_destroy.argtypes = [P]
        lib.ref_h2o_destroy.restype = None
        lib.ref_h2o_observe_attention.argtypes = [P, SZ, SZ, SZ, SZ, P, SZ, C.c_char_p, SZ]
        lib.ref_h2o_observe_group_sums.argtypes = [P, SZ, SZ, SZ, SZ, P, SZ, C.c_char_p, SZ]
        lib.ref_h2o_importance.argtypes = [P, SZ, SZ, SZ, P, C.c_char_p, SZ]
        lib.ref_h2o_resident_ids.argtypes = [P, SZ, P, SZ, P, C.c_char_p, SZ]
        lib.ref_checksum.restype = C.c_uint64
        lib.ref_checksum.argtypes = [P, SZ]
        lib.ref_checksum_four.argtypes = [P, SZ, SZ, P, C.c_char_p, SZ]
        lib.ref_checksum_records.argtypes = [P, P, SZ, SZ, P]
        lib.ref_plan_hot_slots.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, C.c_int, P, P,
                                           C.c_char_p, SZ]
        lib.ref_checksum_records.restype = None
        lib.ref_read_plan.argtypes = [P, SZ, C.c_uint64, C.c_uint64, SZ, SZ, C.c_uint, P, SZ, P, C.c_char_p, SZ]
        lib.ref_segment_roundtrip.argtypes = [C.c_char_p, C.c_uint64, SZ, C.c_uint64, SZ, C.c_uint64, P, P,
                                              C.c_longlong, C.c_ubyte, SZ, P, SZ, P, C.c_char_p, SZ]
        _ref = lib
    return _ref


class OracleError(RuntimeError):
    def __init__(self, code: int, message: str = ""):
        super().__init__(message or f"oracle error {code}")
        self.code = code


# ------------------------------------------------------------------ oracle
def half_bits(x: float) -> int:
    return int(oracle().orc_half_bits(float(x)))


def half_value(h: int) -> float:
    return float(oracle().orc_half_value(int(h)))


def score(q: np.ndarray, k: np.ndarray, n: int, stride: int, threads: int = 8) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    out = np.empty((32, n), dtype=np.uint16)
    rc = oracle().orc_score(_p(q), _p(k), n, stride, _p(out), n, 0, threads)
    if rc:
        raise OracleError(rc)
    return out


def score_views(q: np.ndarray, views: list, threads: int = 8) -> np.ndarray:
    """views: list of (array, first_token_word_offset, tokens, stride)."""
    total = sum(v[2] for v in views)
    out = np.empty((32, total), dtype=np.uint16)
    q = np.ascontiguousarray(q, dtype=np.uint16)
    col = 0
    for arr, off, tokens, stride in views:
        base = arr.ctypes.data + 2 * off
        rc = oracle().orc_score(_p(q), C.c_void_p(base), tokens, stride, _p(out), total, col, threads)
        if rc:
            raise OracleError(rc)
        col += tokens
    return out


def scale(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint16)
    out = np.empty_like(raw)
    oracle().orc_scale(_p(raw), raw.size, _p(out))
    return out


def select(scaled: np.ndarray, heads: int, stride: int, valid: int, alpha: float, ratio: float,
           fp32_counts: bool = False):
    """Returns (ids [heads, k] uint64, counts [heads] uint32, k, tied)."""
    scaled = np.ascontiguousarray(scaled, dtype=np.uint16)
    kcap = max(1, min(int(np.floor(float(valid) * float(np.float32(ratio)))), valid)) if valid else 1
    ids = np.zeros((max(heads, 1), kcap), dtype=np.uint64)
    counts = np.zeros(max(heads, 1), dtype=np.uint32)
    k = C.c_size_t()
    tied = C.c_size_t()
    rc = oracle().orc_select(_p(scaled), heads, stride, valid, C.c_float(alpha), C.c_float(ratio), int(fp32_counts),
                             _p(ids), kcap, _p(counts), C.byref(k), C.byref(tied))
    if rc:
        raise OracleError(rc)
    return ids[:, : k.value], counts, k.value, tied.value


def union(ids: np.ndarray, sizes, visible: int) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.uint64)
    sz = np.ascontiguousarray(sizes, dtype=np.uint64)
    out = np.zeros(max(1, visible), dtype=np.uint64)
    cnt = C.c_size_t()
    rc = oracle().orc_union(_p(ids), ids.shape[1], _p(sz), visible, _p(out), C.byref(cnt))
    if rc:
        raise OracleError(rc)
    return out[: cnt.value]


def pack(ids: np.ndarray, sizes, positions, physical, payload: np.ndarray, count: int):
    ids = np.ascontiguousarray(ids, dtype=np.uint64)
    sz = np.ascontiguousarray(sizes, dtype=np.uint64)
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    phys = np.ascontiguousarray(physical, dtype=np.uint64)
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    qpad = (len(pos) + 63) // 64 * 64
    k = np.empty(count * 4096, dtype=np.uint16)
    v = np.empty(count * 4096, dtype=np.uint16)
    mask = np.empty(count * qpad * 32, dtype=np.float32)
    rc = oracle().orc_pack(_p(ids), ids.shape[1], _p(sz), _p(pos), len(pos), _p(phys), len(phys), _p(payload),
                           payload.size, count, _p(k), _p(v), _p(mask))
    if rc:
        raise OracleError(rc)
    return k, v, mask


def gather_map(prefetched: np.ndarray, prows: int, misses: np.ndarray, mrows: int, row_map: np.ndarray, count: int):
    k = np.empty(count * 4096, dtype=np.uint16)
    v = np.empty(count * 4096, dtype=np.uint16)
    row_map = np.ascontiguousarray(row_map, dtype=np.int32)
    rc = oracle().orc_gather_map(_p(prefetched), prows, _p(misses), mrows, _p(row_map), count, _p(k), _p(v))
    if rc:
        raise OracleError(rc)
    return k, v


def prefetch_cover(raw: np.ndarray, capacity: int, position: int, alpha: float, fp32_counts: bool = False):
    raw = np.ascontiguousarray(raw, dtype=np.uint16)
    cap = min(position, int(np.floor(float(position + 1) * float(np.float32(0.2)))))
    per_head = np.zeros((32, max(cap, 1)), dtype=np.uint64)
    physical = np.zeros(max(position, 1), dtype=np.uint64)
    bound = C.c_size_t()
    nphys = C.c_size_t()
    rc = oracle().orc_prefetch_cover(_p(raw), capacity, position, C.c_float(alpha), int(fp32_counts), _p(per_head),
                                     C.byref(bound), _p(physical), C.byref(nphys))
    if rc:
        raise OracleError(rc)
    return per_head[:, : bound.value], physical[: nphys.value]


def attention_packed(k, v, mask, count: int, qpad: int, q) -> np.ndarray:
    out = np.empty((32, 128), dtype=np.float64)
    q = np.ascontiguousarray(q, dtype=np.float32)
    oracle().orc_attention_packed(_p(k), _p(v), _p(mask), count, qpad, _p(q), _p(out))
    return out


def attention_compact(k, v, count: int, lengths, q) -> np.ndarray:
    out = np.empty((32, 128), dtype=np.float64)
    q = np.ascontiguousarray(q, dtype=np.float32)
    lengths = np.ascontiguousarray(lengths, dtype=np.uint32)
    oracle().orc_attention_compact(_p(k), _p(v), count, _p(lengths), _p(q), _p(out))
    return out


def attention_dense(kc, vc, n: int, stride: int, q) -> np.ndarray:
    out = np.empty((32, 128), dtype=np.float64)
    q = np.ascontiguousarray(q, dtype=np.float32)
    oracle().orc_attention_dense(_p(kc), _p(vc), n, stride, _p(q), _p(out))
    return out


def attention_dense_fast(kc, vc, n: int, q, threads: int) -> np.ndarray:
    """CPU-baseline dense attention (float, threads over heads)."""
    out = np.empty((32, 128), dtype=np.float32)
    oracle().orc_attention_dense_f32(_p(kc), _p(vc), n, 1024, _p(np.ascontiguousarray(q, dtype=np.float32)),
                                     _p(out), threads)
    return out


def attention_packed_fast(k, v, mask, count: int, q, threads: int, qpad: int = 64) -> np.ndarray:
    """CPU-baseline attention over the packed workspace (float)."""
    out = np.empty((32, 128), dtype=np.float32)
    oracle().orc_attention_packed_f32(_p(k), _p(v), _p(mask), count, qpad,
                                      _p(np.ascontiguousarray(q, dtype=np.float32)), _p(out), threads)
    return out


def rehearsal(x_bf16, w_bf16, position: int, theta: float = 500000.0) -> np.ndarray:
    out = np.empty(4096, dtype=np.float64)
    oracle().orc_rehearsal(_p(np.ascontiguousarray(x_bf16, dtype=np.uint16)),
                           _p(np.ascontiguousarray(w_bf16, dtype=np.uint16)), position, theta, _p(out))
    return out


# ------------------------------------------------------------- reference
def synth_normal(count: int, seed: int, stddev: float = 1.0, bf16: bool = False, threads: int = 8) -> np.ndarray:
    """The library's seeded normal generator (hsb_synth_normal_f16/_bf16),
    restated on the CPU: uint16 F16 (or BF16) bits [count]."""
    out = np.empty(count, dtype=np.uint16)
    oracle().orc_synth_normal(_p(out), count, seed, stddev, int(bf16), threads)
    return out


def synth_keys(tokens: int, seed: int, heavy_fraction: float = 0.02, heavy_scale: float = 4.0, rope: bool = True,
               theta: float = 500000.0, stride: int = 1024, threads: int = 8) -> np.ndarray:
    """The library's key-row generator (hsb_synth_keys), restated on the
    CPU: uint16 [tokens * stride] with 1024 words per row written."""
    out = np.zeros(tokens * stride, dtype=np.uint16)
    oracle().orc_synth_keys(_p(out), tokens, stride, seed, heavy_fraction, heavy_scale, int(rope), theta, threads)
    return out


_ref_runtime = None


def ref_runtime_available() -> bool:
    return REF_RUNTIME_SO.exists()


def ref_runtime_decode(rows: np.ndarray, capacity: int, prompt: int, steps: int, layer: int, beta: float,
                       alpha: float, rehearsal: np.ndarray, workdir: str) -> dict:
    """Drives the reference FullGqaRuntimePolicy (oracle/_ref, compiled from
    its sources) through `steps` decode steps of one layer after a prompt of
    `prompt` positions: per step the payload cover its prepare_history
    publishes (full_gqa_runtime.cpp:299-344) and its final selection
    (:549-585).  rows: [capacity][2048] K||V F16 bits; rehearsal: [steps][4096]
    F32 selection queries."""
    global _ref_runtime
    if _ref_runtime is None:
        lib = C.CDLL(str(REF_RUNTIME_SO))
        lib.ref_runtime_decode.argtypes = [C.c_char_p, SZ, SZ, SZ, C.c_int, C.c_double, C.c_float, P, P, P, P, SZ, P,
                                           P, P, SZ, P, P, SZ, C.c_char_p, SZ]
        _ref_runtime = lib
    cap_max = max(1, int(np.floor((prompt + steps + 1) * 0.2)) + 1)
    phys_max, k_max = prompt + steps + 1, cap_max
    rows = np.ascontiguousarray(rows, dtype=np.uint16)
    q = np.ascontiguousarray(rehearsal, dtype=np.float32)
    bound = np.zeros(steps, dtype=np.uint64)
    cover = np.zeros((steps, 32, cap_max), dtype=np.uint64)
    phys = np.zeros((steps, phys_max), dtype=np.uint64)
    nphys = np.zeros(steps, dtype=np.uint64)
    cold = np.zeros((steps, phys_max), dtype=np.uint8)
    k = np.zeros(steps, dtype=np.uint64)
    final = np.zeros((steps, 32, k_max), dtype=np.uint64)
    e = _err()
    if _ref_runtime.ref_runtime_decode(workdir.encode(), capacity, prompt, steps, layer, beta, alpha, _p(rows),
                                       _p(q), _p(bound), _p(cover), cap_max, _p(phys), _p(nphys), _p(cold), phys_max,
                                       _p(k), _p(final), k_max, e, 512):
        raise ReferenceError_(e.value.decode())
    return {"bound": bound, "cover": cover, "physical": phys, "nphysical": nphys, "cold": cold, "k": k,
            "final": final}


def _err():
    return C.create_string_buffer(512)


class ReferenceError_(RuntimeError):
    pass


class RefScorer:
    """The reference FullGqaCpuScorer (implementation 0 automatic, 1 scalar, 2 avx2)."""

    def __init__(self, threads: int, implementation: int = 0):
        e = _err()
        self.h = ref().ref_scorer_create(threads, implementation, e, 512)
        if not self.h:
            raise ReferenceError_(e.value.decode())

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_scorer_destroy(self.h)

    def name(self) -> str:
        return ref().ref_scorer_name(self.h).decode()

    def score(self, q: np.ndarray, views: list) -> np.ndarray:
        """views: list of (array, word offset, tokens, stride)."""
        n = len(views)
        data = (C.c_void_p * max(n, 1))(*[C.c_void_p(a.ctypes.data + 2 * off) for a, off, _, _ in views])
        tokens = (C.c_size_t * max(n, 1))(*[t for _, _, t, _ in views])
        strides = (C.c_size_t * max(n, 1))(*[s for _, _, _, s in views])
        total = sum(t for _, _, t, _ in views)
        out = np.empty((32, max(total, 1)), dtype=np.uint16)
        q = np.ascontiguousarray(q, dtype=np.uint16)
        e = _err()
        if ref().ref_scorer_score(self.h, _p(q), data, tokens, strides, n, _p(out), out.size, e, 512):
            raise ReferenceError_(e.value.decode())
        return out[:, :total]


def ref_select(scaled: np.ndarray, heads: int, stride: int, valid: int, alpha: float, ratio: float,
               fp32_counts: bool = False):
    scaled = np.ascontiguousarray(scaled, dtype=np.uint16)
    kcap = max(1, valid)
    ids = np.zeros((heads, kcap), dtype=np.uint64)
    counts = np.zeros(heads, dtype=np.uint32)
    k = C.c_size_t()
    tied = C.c_size_t()
    e = _err()
    if ref().ref_select(_p(scaled), heads, stride, valid, C.c_float(alpha), C.c_float(ratio), int(fp32_counts),
                        _p(ids), kcap, _p(counts), C.byref(k), C.byref(tied), e, 512):
        raise ReferenceError_(e.value.decode())
    return ids[:, : k.value], counts, k.value, tied.value


def ref_scale(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint16)
    out = np.empty_like(raw)
    ref().ref_scale(_p(raw), raw.size, _p(out))
    return out


def ref_union(ids: np.ndarray, sizes, visible: int) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.uint64)
    sz = np.ascontiguousarray(sizes, dtype=np.uint64)
    out = np.zeros(max(1, visible), dtype=np.uint64)
    cnt = C.c_size_t()
    e = _err()
    if ref().ref_union(_p(ids), ids.shape[1], _p(sz), visible, _p(out), C.byref(cnt), e, 512):
        raise ReferenceError_(e.value.decode())
    return out[: cnt.value]


def ref_pack(ids, sizes, positions, physical, payload, count: int):
    ids = np.ascontiguousarray(ids, dtype=np.uint64)
    sz = np.ascontiguousarray(sizes, dtype=np.uint64)
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    phys = np.ascontiguousarray(physical, dtype=np.uint64)
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    qpad = (len(pos) + 63) // 64 * 64
    k = np.empty(count * 4096, dtype=np.uint16)
    v = np.empty(count * 4096, dtype=np.uint16)
    mask = np.empty(count * qpad * 32, dtype=np.float32)
    e = _err()
    if ref().ref_pack(_p(ids), ids.shape[1], _p(sz), _p(pos), len(pos), _p(phys), len(phys), _p(payload),
                      payload.size, count, _p(k), _p(v), _p(mask), e, 512):
        raise ReferenceError_(e.value.decode())
    return k, v, mask


def h2o_group_sums(buf: np.ndarray, keys: int, queries: int, nb0: int, nb1: int, nb2: int,
                   offset: int = 0) -> np.ndarray:
    """runtime/gqa_h2o_stats.cu:41-57 over the bytes of `buf` (any dtype) from
    byte `offset`: F32 [8][keys] group sums."""
    buf = np.ascontiguousarray(buf)
    need = offset + (keys - 1) * nb0 + (queries - 1) * nb1 + 31 * nb2 + 4
    assert buf.nbytes >= need, "probability buffer too small for the strides"
    out = np.empty((8, keys), dtype=np.float32)
    oracle().orc_h2o_group_sums(C.c_void_p(buf.ctypes.data + offset), keys, queries, nb0, nb1, nb2, _p(out))
    return out


class RefH2O:
    """The reference's H2OResidency (policy/h2o_residency.hpp:16-77)."""

    def __init__(self, layers: int = 1, query_heads: int = 32, kv_heads: int = 8, prompt_tokens: int = 1,
                 generated_capacity: int = 0, prompt_resident: int = 0, budget: int = 1 << 40):
        e = _err()
        self.kv_heads = kv_heads
        self.h = ref().ref_h2o_create(layers, query_heads, kv_heads, prompt_tokens, generated_capacity,
                                      prompt_resident, budget, e, 512)
        if not self.h:
            raise ReferenceError_(e.value.decode())

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_h2o_destroy(self.h)

    def observe_attention(self, layer: int, first: int, queries: int, keys: int, p: np.ndarray) -> None:
        p = np.ascontiguousarray(p, dtype=np.float32)
        e = _err()
        if ref().ref_h2o_observe_attention(self.h, layer, first, queries, keys, _p(p), p.size, e, 512):
            raise ReferenceError_(e.value.decode())

    def observe_group_sums(self, layer: int, first: int, queries: int, keys: int, sums: np.ndarray) -> None:
        sums = np.ascontiguousarray(sums, dtype=np.float32)
        e = _err()
        if ref().ref_h2o_observe_group_sums(self.h, layer, first, queries, keys, _p(sums), sums.size, e, 512):
            raise ReferenceError_(e.value.decode())

    def importance(self, layer: int, count: int) -> np.ndarray:
        out = np.empty((self.kv_heads, count), dtype=np.float32)
        e = _err()
        if ref().ref_h2o_importance(self.h, layer, self.kv_heads, count, _p(out), e, 512):
            raise ReferenceError_(e.value.decode())
        return out

    def resident_ids(self, layer: int, capacity: int) -> list:
        out = np.zeros((self.kv_heads, capacity), dtype=np.uint64)
        sizes = np.zeros(self.kv_heads, dtype=np.uint64)
        e = _err()
        if ref().ref_h2o_resident_ids(self.h, layer, _p(out), capacity, _p(sizes), e, 512):
            raise ReferenceError_(e.value.decode())
        return [out[h, :int(sizes[h])].tolist() for h in range(self.kv_heads)]


# ------------------------------------------------------------ KV records
def fnv1a64(data) -> int:
    b = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray))
                             else data).view(np.uint8)
    return int(oracle().orc_fnv1a64(_p(b), b.nbytes))


def records_encode(payload: np.ndarray, count: int, record_bytes: int, request: int, layer: int, first: int,
                   payload_stride: int | None = None) -> np.ndarray:
    """storage/segmented_store.cpp:95-104: the file image of `count` records."""
    payload = np.ascontiguousarray(payload).view(np.uint8).reshape(-1)
    stride = record_bytes if payload_stride is None else payload_stride
    assert payload.nbytes >= (count - 1) * stride + record_bytes
    out = np.empty(count * (record_bytes + 32), dtype=np.uint8)
    oracle().orc_kv_records_encode(_p(payload), stride, count, record_bytes, request, layer, first, _p(out))
    return out


def records_verify(window: np.ndarray, offsets, positions, request: int, layer: int, record_bytes: int,
                   groups=None, out_rows=None, out_capacity: int | None = None):
    """Returns (code, index, rows [capacity][record_bytes]) walking the
    reference's validation loop (policy/full_gqa_runtime.cpp:394-409)."""
    window = np.ascontiguousarray(window).view(np.uint8).reshape(-1)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    grp = None if groups is None else np.ascontiguousarray(groups, dtype=np.uint32)
    rows = None if out_rows is None else np.ascontiguousarray(out_rows, dtype=np.uint32)
    cap = len(off) if out_capacity is None else out_capacity
    out = np.zeros((max(cap, 1), record_bytes), dtype=np.uint8)
    idx = np.zeros(1, dtype=np.uint32)
    code = oracle().orc_kv_records_verify(_p(window), window.nbytes, _p(off), _p(pos), _p(grp), len(off), request,
                                          layer, record_bytes, _p(out), record_bytes, _p(rows), cap, _p(idx))
    return int(code), int(idx[0]), out[:cap]


def ref_checksum(data: np.ndarray) -> int:
    data = np.ascontiguousarray(data).view(np.uint8)
    return int(ref().ref_checksum(_p(data), data.nbytes))


def ref_checksum_four(rows: list, nbytes: int) -> list:
    arrs = [np.ascontiguousarray(r).view(np.uint8) for r in rows]
    ptrs = (C.c_void_p * 4)(*[a.ctypes.data for a in arrs])
    out = np.zeros(4, dtype=np.uint64)
    e = _err()
    if ref().ref_checksum_four(ptrs, nbytes, len(arrs), _p(out), e, 512):
        raise ReferenceError_(e.value.decode())
    return [int(x) for x in out[:len(arrs)]]


def ref_checksum_records(base: np.ndarray, offsets, nbytes: int) -> np.ndarray:
    """The reference runtime's four-at-a-time digest loop over payloads at
    base + offsets[i] (policy/full_gqa_runtime.cpp:394-408)."""
    base = np.ascontiguousarray(base).view(np.uint8)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    assert len(off) == 0 or int(off.max()) + nbytes <= base.nbytes
    out = np.zeros(len(off), dtype=np.uint64)
    ref().ref_checksum_records(_p(base), _p(off), len(off), nbytes, _p(out))
    return out


def ref_read_plan(offsets, record_bytes: int, extent: int, window_bytes: int = 1 << 20, gap_bytes: int = 16384,
                  amplification: int = 1500) -> np.ndarray:
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    out = np.zeros((max(len(off), 1), 5), dtype=np.uint64)
    n = C.c_size_t(0)
    e = _err()
    if ref().ref_read_plan(_p(off), len(off), record_bytes, extent, window_bytes, gap_bytes, amplification,
                           _p(out), out.shape[0], C.byref(n), e, 512):
        raise ReferenceError_(e.value.decode())
    return out[:n.value]


def ref_segment_roundtrip(path: str, request: int, layers: int, positions: int, record_bytes: int, quota: int,
                          payloads: list, mutate_offset: int = -1, mutate_xor: int = 0, fetch_layer: int = 0,
                          ids=()) -> np.ndarray:
    """The reference SegmentedKVStore writes payloads[l] (rows of layer l from
    position 0) to a new file at `path`, optionally flips one byte, then
    fetches `ids` of `fetch_layer`; returns the fetched bytes."""
    arrs = [np.ascontiguousarray(p).view(np.uint8).reshape(-1) for p in payloads]
    ptrs = (C.c_void_p * layers)(*[a.ctypes.data if a.size else 0 for a in arrs])
    counts = np.array([a.nbytes // record_bytes for a in arrs], dtype=np.uint64)
    want = np.ascontiguousarray(ids, dtype=np.uint64)
    out = np.zeros(max(1, len(want) * record_bytes), dtype=np.uint8)
    e = _err()
    if ref().ref_segment_roundtrip(path.encode(), request, layers, positions, record_bytes, quota, ptrs, _p(counts),
                                   mutate_offset, mutate_xor, fetch_layer, _p(want), len(want), _p(out), e, 512):
        raise ReferenceError_(e.value.decode())
    return out[:len(want) * record_bytes]



def ref_plan_hot_slots(capacity: int, prompt: int, generated: int, beta: float, allow_partial: bool = False):
    """plan_full_gqa_runtime's hot_slot_by_position and prompt hot tokens."""
    out = np.zeros(capacity, dtype=np.int64)
    hot = C.c_uint64(0)
    e = _err()
    if ref().ref_plan_hot_slots(capacity, prompt, generated, beta, int(allow_partial), _p(out), C.byref(hot), e, 512):
        raise ReferenceError_(e.value.decode())
    return out, hot.value
