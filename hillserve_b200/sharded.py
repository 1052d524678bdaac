"""KV-head-sharded selected-KV decode layer over several GPUs.

A batch of independent sequences, each with Q [32,128] and K/V [N,8,128],
runs one selected-KV layer with the 8 KV heads split evenly over the ranks of
a process group: rank r holds KV heads [G r, G (r+1)) with G = 8 / world, i.e.
query heads [4 G r, 4 G (r+1)), of every sequence, as token-major shards
[N][G][128].  The reference couples all heads of a sequence twice
(policy/gqa_policy.cpp:49-63): the threshold comes from query head 0 and k
from the F16 mean of all 32 heads' F16 counts.  A shard step reproduces both
exactly with small exchanges, and then all-gathers the attention outputs:

    1. every rank scores its heads (the rank holding query head 0 also keeps
       head-0 partials);
    2. rank 0 derives each sequence's threshold record -> broadcast;
    3. every rank counts its heads against it -> records all-gathered in head
       order (every rank then folds the same 32 records into the same k);
    4. every rank selects its heads' top-k, gathers their K/V rows into its
       packed buffers and attends over them -> outputs all-gathered.

The sum of F16-rounded integer counts is exact in FP32 in any order, so the
folded k equals the unsharded selector's (policy/full_gqa_runtime.cpp:307-309
makes the same argument).  Phases are methods so that a caller (or a test)
can place the exchanges itself; step() places them with torch.distributed.

PeerExchange does the same exchanges with the library's own kernels over
NVLink peer memory (hsb_exchange_*): every rank's mailbox is mapped into every
process by CUDA IPC, producers store into every mailbox and release an epoch
flag, consumers wait on their own mailbox's flags (bounded waits).  No NCCL
call sits on the data path; the process group only carries the one-time
exchange of IPC handles.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _capi

HEADS, KV_HEADS, DIM = 32, 8, 128


def _ptr(t) -> int:
    return t.data_ptr()


@dataclass
class ShardGeometry:
    world: int
    rank: int

    @property
    def kv_heads(self) -> int:
        return KV_HEADS // self.world

    @property
    def heads(self) -> int:
        return 4 * self.kv_heads

    @property
    def head_base(self) -> int:
        return self.heads * self.rank


def slot_capacity(tokens: int, ratio: float) -> int:
    from . import select_kmax

    return max(32, (select_kmax(tokens, ratio) + 31) // 32 * 32)


class KVHeadShardedLayer:
    """One rank's part of a KV-head-sharded selected-KV layer for `batch`
    sequences of `tokens` tokens.  Device buffers are allocated once."""

    def __init__(self, tokens: int, batch: int, world: int, rank: int, alpha: float = 0.1, ratio: float = 0.2,
                 device="cuda"):
        import torch

        if KV_HEADS % world:
            raise ValueError("world size must divide the 8 KV heads")
        self.torch = torch
        self.geo = ShardGeometry(world, rank)
        self.tokens, self.batch = tokens, batch
        self.alpha, self.ratio = float(alpha), float(ratio)
        self.count = slot_capacity(tokens, ratio)
        h, dev = self.geo.heads, torch.device(device)
        self.lib = _capi.lib()
        u16 = torch.int16
        self.scores = torch.empty((batch, h, tokens), dtype=u16, device=dev)
        self.keys = torch.empty((batch, h, tokens), dtype=u16, device=dev)
        self.head0 = torch.zeros((batch, self.lib.hsb_shard_head0_words()), dtype=torch.int32, device=dev)
        self.thr = torch.zeros((batch, 2), dtype=torch.int32, device=dev)
        self.records = torch.zeros((batch, h), dtype=torch.int32, device=dev)
        self.records_all = torch.zeros((batch, HEADS), dtype=torch.int32, device=dev)
        self.ids = torch.empty((batch, h, self.count), dtype=torch.int32, device=dev)
        self.counts = torch.zeros((batch, h), dtype=torch.int32, device=dev)
        self.results = torch.zeros((batch, 4), dtype=torch.int32, device=dev)
        # The whole batch runs in each kernel: packed K/V per sequence.
        self.k_packed = torch.empty((batch, self.count * h * DIM), dtype=u16, device=dev)
        self.v_packed = torch.empty((batch, self.count * h * DIM), dtype=u16, device=dev)
        self.out = torch.zeros((batch, h, DIM), dtype=torch.float32, device=dev)
        # Outputs and the selection record of each sequence travel together:
        # [batch][heads * 128 + 4] (the record's int32 words bit-cast).
        self.outbox = torch.zeros((batch, h * DIM + 4), dtype=torch.float32, device=dev)
        ws = self.lib.hsb_shard_select_workspace_bytes(self.geo.kv_heads, tokens, self.count, batch)
        self.workspace = torch.empty((ws + 255) // 256 * 256, dtype=torch.uint8, device=dev)

    # ---------------------------------------------------------------- phases
    def _check(self, rc: int, what: str):
        if rc != 0:
            from . import HsbError

            raise HsbError(rc, f"{what}: {self.lib.hsb_last_error().decode()}")

    def score(self, q16, kshard, stream: int):
        """q16 [batch][heads][128] F16 bits, kshard [batch][tokens][G][128]; one launch."""
        owner = self.geo.rank == 0
        self._check(self.lib.hsb_shard_score(_ptr(q16), self.geo.kv_heads, _ptr(kshard), self.tokens, self.batch,
                                             _ptr(self.scores), _ptr(self.keys),
                                             _ptr(self.head0) if owner else None, stream), "shard score")

    def threshold(self, stream: int):
        """Rank 0 only: per-sequence {threshold key, status} records."""
        self._check(self.lib.hsb_shard_threshold(_ptr(self.head0), self.batch, C.c_float(self.alpha),
                                                 _ptr(self.thr), stream), "shard threshold")

    def count_heads(self, stream: int):
        self._check(self.lib.hsb_shard_count(_ptr(self.keys), self.geo.heads, self.tokens, self.batch,
                                             _ptr(self.thr), _ptr(self.records), stream), "shard count")

    def select(self, q32, kshard, vshard, stream: int):
        """q32 [batch][heads][128] F32; uses self.thr and self.records_all."""
        self._check(self.lib.hsb_shard_select(
            _ptr(self.keys), _ptr(self.scores), self.geo.kv_heads, self.tokens, self.batch, _ptr(self.thr),
            _ptr(self.records_all), HEADS, self.geo.head_base, C.c_float(self.alpha), C.c_float(self.ratio),
            _ptr(self.ids), self.count, _ptr(self.counts), _ptr(self.results), _ptr(q32), _ptr(kshard),
            _ptr(vshard), _ptr(self.k_packed), _ptr(self.v_packed), _ptr(self.out), _ptr(self.workspace),
            self.workspace.numel(), stream), "shard select")

    # ------------------------------------------------------- peer memory
    def step_peer(self, q16, q32, kshard, vshard, exchange: PeerExchange, marks=None):
        """The whole layer with the exchanges over peer memory: four launches
        on every rank (rank 0's scorer pushes the thresholds), no collective.  Returns the
        mailbox's outputs [batch][32][128] and the combined selection records
        [batch][4] (k, boundary-tied heads summed over ranks, status code,
        index); the exchange's own status is in exchange.status.  marks: five
        callables run on the current stream around the four phases (event
        records, for a timeline)."""
        torch = self.torch
        stream = torch.cuda.current_stream().cuda_stream
        g = C.byref(exchange.group)
        mark = (lambda i: marks[i]()) if marks else (lambda i: None)
        mark(0)
        if self.geo.rank == 0:  # the scorer pushes the thresholds itself
            self._check(self.lib.hsb_shard_score_push(
                _ptr(q16), self.geo.kv_heads, _ptr(kshard), self.tokens, self.batch, _ptr(self.scores),
                _ptr(self.keys), _ptr(self.head0), C.c_float(self.alpha), g, stream), "shard score push")
        else:
            self.score(q16, kshard, stream)
        mark(1)
        self._check(self.lib.hsb_exchange_count(_ptr(self.keys), self.geo.heads, self.tokens, g, stream),
                    "exchange count")
        mark(2)
        self._check(self.lib.hsb_shard_select(
            _ptr(self.keys), _ptr(self.scores), self.geo.kv_heads, self.tokens, self.batch, exchange.thr_ptr,
            exchange.records_ptr, HEADS, self.geo.head_base, C.c_float(self.alpha), C.c_float(self.ratio),
            _ptr(self.ids), self.count, _ptr(self.counts), _ptr(self.results), _ptr(q32), _ptr(kshard),
            _ptr(vshard), _ptr(self.k_packed), _ptr(self.v_packed), _ptr(self.out), _ptr(self.workspace),
            self.workspace.numel(), stream), "shard select")
        mark(3)
        self._check(self.lib.hsb_exchange_finish(_ptr(self.out), _ptr(self.results), self.geo.heads, g, stream),
                    "exchange finish")
        mark(4)
        res = exchange.results
        combined = res[0].clone()
        combined[:, 1] = res[:, :, 1].sum(dim=0)
        return exchange.outputs, combined

    # ------------------------------------------------------------------ step
    def step(self, q16, q32, kshard, vshard, group=None):
        """The whole layer on this rank; returns the all-gathered outputs
        [batch][32][128] and the combined selection records [batch][4]
        (k, boundary-tied heads summed over ranks, status code, index)."""
        import torch.distributed as dist

        torch = self.torch
        stream = torch.cuda.current_stream().cuda_stream if self.scores.is_cuda else 0
        world = self.geo.world
        self.score(q16, kshard, stream)
        if self.geo.rank == 0:
            self.threshold(stream)
        dist.broadcast(self.thr, src=0, group=group)
        self.count_heads(stream)
        parts = [torch.empty_like(self.records) for _ in range(world)]
        dist.all_gather(parts, self.records, group=group)
        self.records_all.copy_(torch.cat(parts, dim=1))
        self.select(q32, kshard, vshard, stream)
        h = self.geo.heads
        self.outbox[:, :h * DIM].copy_(self.out.view(self.batch, h * DIM))
        self.outbox[:, h * DIM:].copy_(self.results.view(torch.float32))
        boxes = [torch.empty_like(self.outbox) for _ in range(world)]
        dist.all_gather(boxes, self.outbox, group=group)
        out = torch.cat([bx[:, :h * DIM].view(self.batch, h, DIM) for bx in boxes], dim=1)
        res = [bx[:, h * DIM:].contiguous().view(torch.int32) for bx in boxes]
        combined = res[0].clone()
        combined[:, 1] = sum(r[:, 1] for r in res)
        return out, combined


class _DeviceArray:
    """A torch view of library-owned device memory (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """The mailboxes of one KV-head-sharded group over peer memory.

    Every rank creates its mailbox, the IPC handles travel once over the
    process group (all_gather_object), and every rank maps the others'.  The
    mailbox of this rank ends each step with all 32 heads' outputs
    (`outputs`, [batch][32][128] F32) and every rank's selection results."""

    def __init__(self, batch: int, world: int, rank: int, group=None, wait_limit_ns: int = 0):
        import torch

        self.lib = _capi.lib()
        self.batch, self.world, self.rank = batch, world, rank
        self.layout = _capi.MailboxLayout()
        self.lib.hsb_mailbox_layout_of(batch, C.byref(self.layout))
        handle = (C.c_ubyte * 64)()
        own = C.c_void_p()
        self._check(self.lib.hsb_mailbox_create(batch, C.byref(own), handle), "mailbox create")
        self.own = own.value
        self.opened = []
        ptrs = [0] * world
        ptrs[rank] = self.own
        if world > 1:
            import torch.distributed as dist

            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            for w in range(world):
                if w == rank:
                    continue
                peer = C.c_void_p()
                buf = (C.c_ubyte * 64).from_buffer_copy(handles[w])
                self._check(self.lib.hsb_mailbox_open(buf, C.byref(peer)), f"mailbox open (rank {w})")
                ptrs[w] = peer.value
                self.opened.append(peer.value)
        self.group = _capi.PeerGroup()
        self.group.world, self.group.rank, self.group.batch = world, rank, batch
        self.group.wait_limit_ns = int(wait_limit_ns)
        for w in range(world):
            self.group.mailbox[w] = ptrs[w]
        lay = self.layout
        self.outputs = torch.as_tensor(_DeviceArray(self.own + lay.outputs, (batch, HEADS, DIM), "<f4"),
                                       device="cuda")
        self.results = torch.as_tensor(_DeviceArray(self.own + lay.results, (world, batch, 4), "<i4"),
                                       device="cuda")
        self.status = torch.as_tensor(_DeviceArray(self.own + lay.status, (2,), "<i4"), device="cuda")
        self.thr_ptr = self.own + lay.thr
        self.records_ptr = self.own + lay.records

    def _check(self, rc: int, what: str):
        if rc != 0:
            from . import HsbError

            raise HsbError(rc, f"{what}: {self.lib.hsb_last_error().decode()}")

    def close(self):
        """Unmaps the peers' mailboxes and frees this rank's (after the
        group's last step; every rank calls it)."""
        for p in self.opened:
            self.lib.hsb_mailbox_close(C.c_void_p(p))
        self.opened = []
        if self.own:
            self.lib.hsb_mailbox_destroy(C.c_void_p(self.own))
            self.own = 0


def shard_rows(full, world: int, rank: int):
    """[batch][tokens][8][128] -> this rank's contiguous [batch][tokens][G][128]."""
    g = KV_HEADS // world
    return full[:, :, g * rank:g * (rank + 1), :].contiguous()


def shard_queries(full, world: int, rank: int):
    """[batch][32][128] -> this rank's [batch][4G][128]."""
    h = HEADS // world
    return full[:, h * rank:h * (rank + 1), :].contiguous()
