"""Batch-sharded data-parallel inference across the GPUs of one node.

The reference has no distributed code (README roadmap "Multi-GPU via NCCL",
README.md:625). Sequences are independent, so the batch is split across
ranks (one process per GPU): rank r owns rows [lo_r, hi_r), holds a full
weight replica and its own KV-cache slice, and runs prefill / decode with no
collective in the data path. The only collective is an all_gather of the
generated tokens (or last-position logits) when the caller needs the whole
batch on every rank. Every collective runs under the process-group timeout
given at init, so a rank that never joins ends the others' call with an
error instead of a hang.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Rows [lo, hi) of a batch owned by `rank`; the first batch % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_batch(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    lo, hi = shard_range(x.shape[0], rank, world)
    return x[lo:hi]


def gather_batch(local: torch.Tensor, batch: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gathers per-rank row shards (shapes from shard_range) into the full [batch, ...] tensor.

    Uneven shards are padded to the largest shard for the collective and
    trimmed afterwards.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_range(batch, rank, world)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank}: local shard has {local.shape[0]} rows, expected {hi - lo}")
    rows = -(-batch // world)
    buf = local.new_zeros((rows, *local.shape[1:]))
    buf[: local.shape[0]] = local
    out = local.new_empty((rows * world, *local.shape[1:]))
    dist.all_gather_into_tensor(out, buf.contiguous(), group=group)
    parts = []
    for r in range(world):
        a, b = shard_range(batch, r, world)
        parts.append(out[r * rows: r * rows + (b - a)])
    return torch.cat(parts, dim=0)


def init_from_env(backend: Optional[str] = None, timeout_s: float = 120.0) -> Tuple[int, int, int]:
    """Initialises the default process group from torchrun's env; returns (rank, world, local_rank).

    With WORLD_SIZE unset (or 1) no process group is created.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class ShardedGPT:
    """Runs one CutileGPT replica per rank on its slice of the batch."""

    def __init__(self, model, group: Optional[dist.ProcessGroup] = None):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        # With time_gather set (and CUDA tensors), CUDA events bracket every all_gather on the
        # current stream; gather_ms() returns the device time of the gathers since the last reset.
        self.time_gather = False
        self._gather_events = []

    def _gather(self, local: torch.Tensor, batch: int) -> torch.Tensor:
        if not (self.time_gather and local.is_cuda):
            return gather_batch(local, batch, self.group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = gather_batch(local, batch, self.group)
        e1.record()
        self._gather_events.append((e0, e1))
        return out

    def gather_ms(self, reset: bool = True) -> float:
        """Device time (ms) of the gathers recorded since the last reset (synchronises on them)."""
        total = 0.0
        for e0, e1 in self._gather_events:
            e1.synchronize()
            total += e0.elapsed_time(e1)
        if reset:
            self._gather_events = []
        return total

    def local_rows(self, batch: int) -> Tuple[int, int]:
        return shard_range(batch, self.rank, self.world)

    def generate(self, idx: torch.Tensor, max_new_tokens: int, gather: bool = True, **kw) -> torch.Tensor:
        """Greedy/sampled generation of this rank's rows; all ranks get the full batch if gather."""
        B = idx.shape[0]
        lo, hi = self.local_rows(B)
        out = self.model.generate(idx[lo:hi], max_new_tokens, **kw)
        if not gather or self.world == 1:
            return out
        return self._gather(out, B)

    def forward_last(self, idx: torch.Tensor, gather: bool = True) -> torch.Tensor:
        """Last-position logits of this rank's rows (gathered to [B, V] if requested)."""
        B = idx.shape[0]
        lo, hi = self.local_rows(B)
        logits = self.model.forward_last(idx[lo:hi])
        if not gather or self.world == 1:
            return logits
        return self._gather(logits, B)

    def forward_gather_last(self, idx: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """The full forward of this rank's rows (logits at every position, as CutileGPT.forward) and
        the last-position logits of the whole batch gathered on every rank: ([b, T, V], [B, V])."""
        B = idx.shape[0]
        lo, hi = self.local_rows(B)
        logits, _ = self.model(idx[lo:hi])
        last = logits[:, -1, :].contiguous()
        return logits, (last if self.world == 1 else self._gather(last, B))
