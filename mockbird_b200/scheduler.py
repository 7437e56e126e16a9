"""Stream scheduler: shard independent synthesis streams across the GPUs of a box.

The reference synthesises one utterance at a time on one device (the engine is
stateful and single-stream, gpu.ts:120-122; the frame loop is sequential,
runtime.ts:540).  Streams share no state, so the multi-GPU build shards them: one
process per GPU, each owning the rings of its streams, with no collective on the
decode path.  torch.distributed (NCCL between GPUs, gloo on CPU) only gathers the
per-rank results for reporting.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    streams: np.ndarray  # global stream ids owned by this rank, ascending

    @property
    def count(self) -> int:
        return int(self.streams.size)


def partition_streams(total: int, world: int, lengths=None) -> list[Shard]:
    """Split `total` stream ids over `world` ranks.

    Without `lengths`: contiguous, equal-size blocks (the first `total % world`
    ranks take one extra stream).  With per-stream live lengths: greedy
    longest-first assignment to the rank with the least total length, so that
    the bytes each rank streams per decode step (proportional to the sum of live
    lengths) are balanced; ties go to the lower rank, and every rank ends up with
    a count within one of total / world.
    """
    if total < 0 or world <= 0:
        raise ValueError("total must be >= 0 and world > 0")
    if lengths is None:
        base, extra = divmod(total, world)
        out, start = [], 0
        for r in range(world):
            n = base + (1 if r < extra else 0)
            out.append(Shard(r, world, np.arange(start, start + n, dtype=np.int32)))
            start += n
        return out
    lengths = np.asarray(lengths, dtype=np.int64)
    if lengths.shape != (total,):
        raise ValueError("lengths must have one entry per stream")
    cap = -(-total // world)  # ceil: keeps per-rank counts balanced
    load = np.zeros(world, np.int64)
    count = np.zeros(world, np.int64)
    owner = np.empty(total, np.int64)
    for sid in np.argsort(-lengths, kind="stable"):
        open_ranks = np.flatnonzero(count < cap)
        r = int(open_ranks[np.argmin(load[open_ranks])])
        owner[sid] = r
        load[r] += lengths[sid]
        count[r] += 1
    return [Shard(r, world, np.flatnonzero(owner == r).astype(np.int32)) for r in range(world)]


def dist_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (defaults 0, 1, 0)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def init_group(backend: str, timeout_s: float = 120.0, device=None):
    """Initialise the default process group from the environment (127.0.0.1 rendezvous).

    `device`: this rank's CUDA device (NCCL binds the group to it)."""
    import torch.distributed as dist

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    rank, world, _ = dist_env()
    if not dist.is_initialized():
        kw = {"device_id": device} if device is not None else {}
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist


def gather_reports(report: dict, device=None) -> list[dict]:
    """All-gather one small dict per rank (reporting only; never on the decode path)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [report]
    keys = sorted(report)
    vals = torch.tensor([float(report[k]) for k in keys], dtype=torch.float64,
                        device=device if device is not None else "cpu")
    out = [torch.empty_like(vals) for _ in range(dist.get_world_size())]
    dist.all_gather(out, vals)
    return [dict(zip(keys, t.tolist())) for t in out]


def max_over_ranks(value: float, device=None) -> float:
    """Max of a scalar over all ranks (the timing rule: a step takes as long as its slowest rank)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
