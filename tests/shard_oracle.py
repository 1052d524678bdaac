"""Numpy restatements of the KV-head shard phases (test oracle only).

Used by the sharded-layer tests: the CPU protocol test swaps them in for the
CUDA phases of hillserve_b200.sharded.KVHeadShardedLayer, and both tests
compare the sharded result with the unsharded reference path (the oracle's
score + scale + select, policy/gqa_policy.cpp:47-70, and attention over the
selected rows, runtime/gqa_delivery.cpp:19-20)."""
from __future__ import annotations

import math

import numpy as np

HEADS, KV, DIM = 32, 8, 128
E_ZERO = 70


def order_keys(bits: np.ndarray) -> np.ndarray:
    """policy/half_order.hpp:7-10 over F16 bit patterns (-0 == +0)."""
    b = bits.astype(np.uint32)
    b = np.where((b & 0x7FFF) == 0, 0, b)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b ^ 0x8000).astype(np.uint32)


def key_nan(k):
    return (k > 0xFC00) | (k < 0x03FF)


def key_nonfinite(k):
    return (k >= 0xFC00) | (k <= 0x03FF)


def key_to_half(key: int) -> np.float16:
    bits = (key ^ 0x8000) if key & 0x8000 else (~key & 0xFFFF)
    return np.array([bits], dtype=np.uint16).view(np.float16)[0]


def threshold_record(keys0: np.ndarray, alpha: float):
    """{threshold key, status} from query head 0's keys (gqa_policy.cpp:49-54)."""
    finite = ~key_nan(keys0)
    if np.any(key_nonfinite(keys0)):
        return 0, 22
    mx = int(keys0[finite].max()) if np.any(finite) else 0
    maximum = np.float32(key_to_half(mx)) if mx else np.float32(-np.inf)
    thr = np.float16(maximum - np.float32(alpha))
    if not np.isfinite(thr):
        return 0, 23
    return int(order_keys(np.array([thr]).view(np.uint16))[0]), 0


def count_records(keys: np.ndarray, thr_key: int) -> np.ndarray:
    """One record per head: count of keys >= thr (NaN excluded) | non-finite << 31."""
    out = np.zeros(keys.shape[0], dtype=np.uint32)
    for h in range(keys.shape[0]):
        k = keys[h]
        c = int(np.count_nonzero(~key_nan(k) & (k >= thr_key)))
        out[h] = c | (int(np.any(key_nonfinite(k))) << 31)
    return out


def fold(records: np.ndarray, n: int, ratio: float):
    """k and status from all heads' records (gqa_policy.cpp:55-63)."""
    total = np.float32(0)
    for h, rec in enumerate(records.astype(np.uint64)):
        c, bad = int(rec & 0x7FFFFFFF), int(rec >> 31)
        if bad:
            return 0, 24, h
        r = np.float16(c)
        if not np.isfinite(r):
            return 0, 26, h
        total = np.float32(total + np.float32(r))
    mean = np.float16(np.float32(total) / np.float32(len(records)))
    if not np.isfinite(mean):
        return 0, 27, 0
    k = min(int(math.floor(float(mean))), int(math.floor(n * float(np.float32(ratio)))), n)
    return k, (E_ZERO if k == 0 else 0), 0


def topk(keys_row: np.ndarray, k: int) -> np.ndarray:
    """First k ids by (key descending, id ascending)."""
    order = np.lexsort((np.arange(keys_row.size), -keys_row.astype(np.int64)))
    return order[:k].astype(np.uint32)


def attention(q32: np.ndarray, krows: np.ndarray, vrows: np.ndarray) -> np.ndarray:
    """softmax(K.q / sqrt(128)) . V in double precision (one query head)."""
    if krows.shape[0] == 0:
        return np.zeros(DIM)
    s = krows.astype(np.float64) @ q32.astype(np.float64) / math.sqrt(DIM)
    w = np.exp(s - s.max())
    return (w / w.sum()) @ vrows.astype(np.float64)


def unsharded(ob, q16: np.ndarray, q32: np.ndarray, k: np.ndarray, v: np.ndarray, n: int, alpha: float,
              ratio: float = 0.2):
    """The reference path for one sequence: ids [32][k], counts, k, ties, out [32][128].
    k, v: F16 bits [n][8][128]."""
    raw = ob.score(q16.reshape(-1), k.reshape(-1), n, 1024)
    scaled = ob.scale(raw)
    ids, counts, kk, tied = ob.select(scaled, HEADS, n, n, alpha, ratio)
    kf = k.view(np.float16).reshape(n, KV, DIM)
    vf = v.view(np.float16).reshape(n, KV, DIM)
    out = np.zeros((HEADS, DIM))
    for h in range(HEADS):
        sel = np.asarray(ids[h][:kk], dtype=np.int64) if kk else np.zeros(0, dtype=np.int64)
        out[h] = attention(q32[h], kf[sel, h // 4, :], vf[sel, h // 4, :])
    return ids, counts, kk, tied, out, scaled
