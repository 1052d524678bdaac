"""The KV-head shard exchange on CPU: two gloo ranks run
KVHeadShardedLayer.step() -- threshold broadcast, count-record all-gather in
head order, output and record all-gathers -- with the four device phases
swapped for numpy restatements (tests/shard_oracle.py), and rank 0 checks the
result against the unsharded reference path."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_oracle_layer():
    import torch

    import shard_oracle as so
    from hillserve_b200 import sharded as sh
    from oracle import binding as ob

    class OracleShard(sh.KVHeadShardedLayer):
        """The shard phases restated on the CPU (test only)."""

        def score(self, q16, kshard, stream):
            g, lo = self.geo.kv_heads, self.geo.head_base
            self.scaled = []
            for b in range(self.batch):
                kfull = np.zeros((self.tokens, 8, 128), dtype=np.uint16)
                kfull[:, lo // 4:lo // 4 + g, :] = kshard[b].numpy().view(np.uint16)
                qfull = np.zeros((32, 128), dtype=np.uint16)
                qfull[lo:lo + self.geo.heads] = q16[b].numpy().view(np.uint16)
                raw = ob.score(qfull.reshape(-1), kfull.reshape(-1), self.tokens, 1024)[lo:lo + self.geo.heads]
                scaled = ob.scale(raw)
                self.scaled.append(scaled)
                self.scores[b].copy_(torch.from_numpy(raw.view(np.int16)))
                self.keys[b].copy_(torch.from_numpy(so.order_keys(scaled).astype(np.uint16).view(np.int16)))

        def threshold(self, stream):
            for b in range(self.batch):
                keys0 = self.keys[b][0].numpy().view(np.uint16).astype(np.uint32)
                key, status = so.threshold_record(keys0, self.alpha)
                self.thr[b] = torch.tensor([key, status], dtype=torch.int32)

        def count_heads(self, stream):
            for b in range(self.batch):
                keys = self.keys[b].numpy().view(np.uint16).astype(np.uint32)
                rec = so.count_records(keys, int(self.thr[b][0]))
                self.records[b].copy_(torch.from_numpy(rec.view(np.int32)))

        def select(self, q32, kshard, vshard, stream):
            n, h = self.tokens, self.geo.heads
            for b in range(self.batch):
                self.out[b].zero_()
                status = int(self.thr[b][1])
                if status:
                    self.results[b] = torch.tensor([0, 0, status, 0], dtype=torch.int32)
                    continue
                rec = self.records_all[b].numpy().view(np.uint32)
                k, status, index = so.fold(rec, n, self.ratio)
                self.counts[b].copy_(torch.from_numpy((rec[self.geo.head_base:self.geo.head_base + h]
                                                       & 0x7FFFFFFF).astype(np.int32)))
                ties = 0
                keys = self.keys[b].numpy().view(np.uint16).astype(np.uint32)
                kf = kshard[b].numpy().view(np.float16)
                vf = vshard[b].numpy().view(np.float16)
                for j in range(h):
                    order = so.topk(keys[j], n)
                    sel = order[:k]
                    self.ids[b][j, :k] = torch.from_numpy(sel.astype(np.int32))
                    if 0 < k < n and self.scaled[b][j][order[k - 1]] == self.scaled[b][j][order[k]]:
                        ties += 1
                    if k:
                        out = so.attention(q32[b][j].numpy(), kf[sel.astype(np.int64), j // 4, :],
                                           vf[sel.astype(np.int64), j // 4, :])
                        self.out[b][j] = torch.from_numpy(out.astype(np.float32))
                self.results[b] = torch.tensor([k, ties, status, index], dtype=torch.int32)

    return OracleShard


def _worker(rank, port, n, batch, alpha, q16, k, v, out_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from hillserve_b200 import sharded as sh

        layer = _make_oracle_layer()(n, batch, WORLD, rank, alpha=alpha, device="cpu")
        q16t = torch.from_numpy(q16.view(np.int16))
        q32t = torch.from_numpy(q16.view(np.float16).astype(np.float32))
        kt = torch.from_numpy(k.view(np.int16))
        vt = torch.from_numpy(v.view(np.int16))
        out, res = layer.step(sh.shard_queries(q16t, WORLD, rank), sh.shard_queries(q32t, WORLD, rank),
                              sh.shard_rows(kt, WORLD, rank), sh.shard_rows(vt, WORLD, rank))
        if rank == 0:
            np.savez(out_path, out=out.numpy(), res=res.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("alpha", [10.0, 0.1])
def test_two_rank_exchange_matches_unsharded(ob, tmp_path, alpha):
    import torch.multiprocessing as mp

    import inputs
    import shard_oracle as so

    n, batch = 512, 2
    q16 = np.stack([inputs.config1(n, seed=60 + b)[0].reshape(32, 128) for b in range(batch)])
    k = np.stack([inputs.config1(n, seed=60 + b)[1].reshape(n, 8, 128) for b in range(batch)])
    v = np.stack([inputs.values(60 + b, n).reshape(n, 8, 128) for b in range(batch)])
    out_path = str(tmp_path / "rank0.npz")
    mp.spawn(_worker, args=(_free_port(), n, batch, alpha, q16, k, v, out_path), nprocs=WORLD, join=True)
    got = np.load(out_path)
    for b in range(batch):
        q32 = q16[b].view(np.float16).astype(np.float32)
        ids, counts, kk, tied, out, _ = so.unsharded(ob, q16[b], q32, k[b], v[b], n, alpha)
        assert got["res"][b][0] == kk
        assert got["res"][b][1] == tied
        assert got["res"][b][2] == (so.E_ZERO if kk == 0 else 0)
        np.testing.assert_allclose(got["out"][b], out, rtol=0, atol=1e-5 * max(1.0, np.abs(out).max()))
