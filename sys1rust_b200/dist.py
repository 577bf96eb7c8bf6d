"""Multi-GPU plumbing of the forward: one process per GPU, weights replicated, requests sharded.

Requests are independent, so the path shards with no collective on the data path (the reference
serves one request at a time on one device, ``runtime/crates/sys1rust/src/worker.rs:1-4``; here
each rank serves its own share). A rank's share is its slice of a longest-first, least-loaded
assignment by token count (``workloads.shard_lpt``), which every rank computes identically from
the same request stream, so no request lists are exchanged. The only collectives are the step
barrier and the max-over-ranks reduction of timings: NCCL between GPUs, gloo on CPU (the tests).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Sequence

from .batch import EncodedItem
from .workloads import shard_lpt


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local: int


def env_rank() -> RankInfo:
    """RANK / WORLD_SIZE / LOCAL_RANK as set by torch.distributed.run (defaults: one process)."""
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def shard_for_rank(requests: Sequence[EncodedItem], world: int, rank: int) -> List[EncodedItem]:
    """This rank's requests, in arrival order. Every request belongs to exactly one rank."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return shard_lpt(list(requests), world)[rank]


def init(world: int, backend: str = "nccl", timeout_s: float = 120.0, device=None) -> None:
    """Join the process group (no-op for one process). A short timeout makes a rank that never
    arrives end the others' next collective with an error instead of a hang."""
    if world <= 1:
        return
    import torch.distributed as dist
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device=None) -> float:
    """The largest value of ``x`` over all ranks (a device time: the slowest rank sets the job)."""
    if world <= 1:
        return float(x)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device=None) -> float:
    if world <= 1:
        return float(x)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_over_ranks(values, world: int, rank: int, device=None) -> list:
    """Every rank's ``values`` (a list of floats of the same length on every rank), as a list
    indexed by rank: one summing all-reduce of a [world, len] table each rank fills one row of."""
    if world <= 1:
        return [list(map(float, values))]
    import torch
    import torch.distributed as dist
    t = torch.zeros(world, len(values), dtype=torch.float64, device=device)
    t[rank] = torch.tensor([float(v) for v in values], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().tolist()


def shutdown(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
