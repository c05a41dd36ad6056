"""Multi-GPU layer of the RDT-1B path: robot sessions sharded across ranks.

One process per GPU (torchrun). Every rank serves its own sessions with its
own model, condition K/V cache and CUDA graph, so nothing crosses ranks on the
data path: the path partitions by session, and there is no exchange step to
put a collective on (the reference serves one robot per process,
include/servoflow/runtime/ and src/sampling/flow_matching.cpp:25-93 have no
multi-GPU code). The only collectives are the barrier around a timed region
and the max over ranks of device-timed statistics.

Rank r owns the global sessions [r·per_rank, (r+1)·per_rank); a session's
seeds derive from its global id, so the same session gets the same weights and
inputs whatever the world size.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Sequence


@dataclass(frozen=True)
class RankInfo:
    world: int
    rank: int
    local: int


def rank_env() -> RankInfo:
    """World size, rank and local rank from torchrun's environment (1, 0, 0 alone)."""
    return RankInfo(int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def session_ids(world: int, rank: int, per_rank: int) -> range:
    """Global ids of the sessions rank `rank` serves (weak scaling: per_rank fixed)."""
    if world < 1 or not 0 <= rank < world or per_rank < 1:
        raise ValueError(f"bad shard: world {world}, rank {rank}, per_rank {per_rank}")
    return range(rank * per_rank, (rank + 1) * per_rank)


def session_seed(session: int, stream: str) -> int:
    """Seed of one session's random stream: "weights", "inputs" or "serving"."""
    base = {"weights": 1000, "inputs": 2000, "serving": 3000}[stream]
    return base + session


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


def barrier() -> None:
    """Barrier over all ranks (no-op alone)."""
    d = _dist()
    if d is not None and d.get_world_size() > 1:
        d.barrier()


def max_over_ranks(values: Sequence[float], device=None) -> List[float]:
    """Element-wise max over ranks of device-timed statistics (identity
    alone). `device` is where the reduction tensor lives: the rank's GPU under
    NCCL, the CPU under gloo."""
    import torch
    d = _dist()
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if d is not None and d.get_world_size() > 1:
        d.all_reduce(t, op=d.ReduceOp.MAX)
    return t.tolist()
