"""Batch sharding across ranks (cutilegpt_b200/distributed.py), tested with gloo ranks on the CPU.

The data path has no collective; only the final all_gather of tokens / logits
crosses ranks. A rank that fails before the gather must make the others'
gather fail within the process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cutilegpt_b200.distributed import ShardedGPT, gather_batch, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_partitions_batch():
    for B in (1, 5, 8, 64, 63):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                lo, hi = shard_range(B, r, world)
                assert 0 <= lo <= hi <= B
                rows += list(range(lo, hi))
            assert rows == list(range(B))
            sizes = [shard_range(B, r, world)[1] - shard_range(B, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


class _FakeModel:
    """Stands in for CutileGPT on the CPU: appends (row id * 10 + step) tokens."""

    def generate(self, idx, n, **kw):
        steps = torch.arange(n).view(1, n) + idx[:, :1] * 10
        return torch.cat([idx, steps], dim=1)

    def forward_last(self, idx):
        return idx.float().sum(dim=1, keepdim=True).repeat(1, 3)


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        B = 5
        full = torch.arange(B).view(B, 1).repeat(1, 3)
        if mode == "gather":
            lo, hi = shard_range(B, rank, world)
            got = gather_batch(full[lo:hi] * 2, B)
            q.put((rank, "ok", torch.equal(got, full * 2)))
        elif mode == "sharded":
            sg = ShardedGPT(_FakeModel())
            out = sg.generate(full, 4)
            ref = _FakeModel().generate(full, 4)
            logits = sg.forward_last(full)
            q.put((rank, "ok", torch.equal(out, ref) and torch.equal(logits, _FakeModel().forward_last(full))))
        elif mode == "dead_rank":
            if rank == 1:
                q.put((rank, "exited", None))
                q.close()
                q.join_thread()        # flush the message, then leave without joining the collective
                os._exit(0)
            lo, hi = shard_range(B, rank, world)
            try:
                gather_batch(full[lo:hi], B)
                q.put((rank, "ok", False))
            except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
                q.put((rank, "error", type(e).__name__))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, val = q.get(timeout=timeout)
        results[rank] = (status, val)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def test_gather_batch_uneven_shards():
    res = _run("gather")
    assert all(v == ("ok", True) for v in res.values()), res


def test_sharded_generate_and_logits_match_unsharded():
    res = _run("sharded")
    assert all(v == ("ok", True) for v in res.values()), res


def test_rank_that_never_joins_fails_the_gather_instead_of_hanging():
    res = _run("dead_rank")
    assert res[1][0] == "exited"
    assert res[0][0] == "error", res
