"""KV-head shards on 2, 4 or 8 GPUs with the exchanges over peer memory.

One process per GPU (torch.multiprocessing, NCCL process group only for the
one-time IPC-handle exchange and a barrier); each rank runs steps of the
sharded layer through hsb_exchange_* and checks, against the unsharded
reference path computed on the CPU, that its mailbox holds every head's
output and every rank's selection results: k, boundary ties and status equal
the reference's, outputs within 2e-3.  Skipped with fewer than two GPUs.
NVLS stays off; the kernels use plain peer stores."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
TOL = 2e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, n: int, batch: int, alpha: float, queue):
    for p in (str(ROOT), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch
    import torch.distributed as dist

    import inputs
    from hillserve_b200 import sharded as sh

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ex = None
    try:
        qs, ks, vs = [], [], []
        for b in range(batch):
            q16, k, _ = inputs.config1(n, seed=300 + b)
            qs.append(q16.reshape(32, 128))
            ks.append(k.reshape(n, 8, 128))
            vs.append(inputs.values(300 + b, n).reshape(n, 8, 128))
        q16 = np.stack(qs)
        dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dt).cuda()  # noqa: E731
        q16t = dev(q16.view(np.int16), torch.int16)
        q32t = dev(q16.view(np.float16).astype(np.float32), torch.float32)
        kt, vt = dev(np.stack(ks).view(np.int16), torch.int16), dev(np.stack(vs).view(np.int16), torch.int16)
        layer = sh.KVHeadShardedLayer(n, batch, world, rank, alpha=alpha)
        ex = sh.PeerExchange(batch, world, rank, wait_limit_ns=2_000_000_000)
        q16l, q32l = sh.shard_queries(q16t, world, rank), sh.shard_queries(q32t, world, rank)
        kl, vl = sh.shard_rows(kt, world, rank), sh.shard_rows(vt, world, rank)
        results = []
        for _ in range(3):
            out, res = layer.step_peer(q16l, q32l, kl, vl, ex)
            torch.cuda.synchronize()
            results.append((out.cpu().numpy().copy(), res.cpu().numpy().copy()))
        status = ex.status.cpu().numpy().copy()
        dist.barrier()
        queue.put((rank, status, results))
    except Exception as e:  # reported to the parent, which fails the test
        queue.put((rank, None, repr(e)))
    finally:
        if ex is not None:
            torch.cuda.synchronize()
            dist.barrier()  # every rank is done with the peers' mailboxes before they are freed
            ex.close()
        dist.destroy_process_group()


def _gpus() -> int:
    torch = pytest.importorskip("torch")
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange_across_gpus(ob, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    import inputs
    import shard_oracle as so

    n, batch, alpha = 4096, 4, 10.0
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, batch, alpha, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=300)
        got[rank] = (status, payload)
    for p in procs:
        p.join(timeout=120)
    for rank in range(world):
        status, payload = got[rank]
        assert status is not None, f"rank {rank}: {payload}"
        assert status[0] == 0, (rank, status)
    want = []
    for b in range(batch):
        q16, k, _ = inputs.config1(n, seed=300 + b)
        v = inputs.values(300 + b, n)
        q32 = q16.view(np.float16).astype(np.float32)
        want.append(so.unsharded(ob, q16.reshape(32, 128), q32.reshape(32, 128), k.reshape(n, 8, 128),
                                 v.reshape(n, 8, 128), n, alpha))
    for rank in range(world):
        for out, res in got[rank][1]:
            for b in range(batch):
                ids, counts, kk, tied, wout, _ = want[b]
                assert res[b, 0] == kk and res[b, 1] == tied, (rank, b, res[b], kk, tied)
                assert res[b, 2] == (so.E_ZERO if kk == 0 else 0)
                o = out[b].astype(np.float64)
                if kk == 0:
                    assert np.all(o == 0.0)
                else:
                    assert np.max(np.abs(o - wout)) <= TOL * np.max(np.abs(wout)), (rank, b)
