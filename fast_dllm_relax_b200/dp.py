"""Data-parallel serving by request: one process per GPU, no collective on the decode path.

Requests are independent (each owns its prompt and KV cache), so a job of n requests is cut into
contiguous ranges, one per rank, and every rank decodes its range with its own library handle
and a full replica of the 3.09 GB of weights.  The only collectives are off the decode path:
the max-over-ranks of the device-timed seconds and the sum of generated tokens after the timed
region, and an optional gather of the outputs to rank 0.  Works over NCCL (GPU tensors) and
gloo (CPU tensors); the host logic is tested on CPU with gloo ranks.
"""

from __future__ import annotations

import os
from typing import Any, Callable, Sequence

import torch
import torch.distributed as dist


def world_info() -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment (1, 0, 0 when absent)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def request_range(n_requests: int, world: int, rank: int) -> range:
    """Contiguous, balanced slice of [0, n_requests) for `rank`: the first n % world ranks take
    one request more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_requests < 0:
        raise ValueError("n_requests must be non-negative")
    base, extra = divmod(n_requests, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def serve(requests: Sequence[Any], decode: Callable[[Any], Any], world: int, rank: int) -> list[tuple[int, Any]]:
    """Decode this rank's slice of `requests`; returns (request index, result) pairs."""
    return [(i, decode(requests[i])) for i in request_range(len(requests), world, rank)]


def reduce_max_sum(maxes: Sequence[float], sums: Sequence[float], device: torch.device | str = "cpu",
                   group=None) -> tuple[list[float], list[float]]:
    """All-reduce `maxes` with MAX and `sums` with SUM (float64), both in the same order on every
    rank.  A no-op without an initialised process group."""
    mx = torch.tensor(list(maxes), dtype=torch.float64, device=device)
    sm = torch.tensor(list(sums), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM, group=group)
    return mx.tolist(), sm.tolist()


def gather_results(local: list[tuple[int, Any]], n_requests: int, group=None) -> list[Any] | None:
    """Collect every rank's (index, result) pairs on rank 0, ordered by request index; other
    ranks get None.  Off the decode path (pickled objects)."""
    if not (dist.is_available() and dist.is_initialized()):
        out = [None] * n_requests
        for i, r in local:
            out[i] = r
        return out
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    parts = [None] * world if rank == 0 else None
    dist.gather_object(local, parts, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_requests
    for part in parts:
        for i, r in part:
            out[i] = r
    return out
