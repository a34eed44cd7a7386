"""Request-level sharding across GPUs for the dual-AR decode path.

Utterances are independent (src/s2_generate.cpp:11-216 runs one utterance
per call), so N GPUs decode N utterances at once with no data exchange: rank
r owns utterance r, its own weight replica, sequence and stream.  The only
collectives are for measurement: a barrier around the timed region and the
maximum of the per-rank device times (the job takes as long as its slowest
rank).  Works with any torch.distributed backend (nccl on GPUs, gloo on CPU).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def dist_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def init(backend: str, local_rank: int, timeout_s: float = 300.0) -> None:
    """Join the process group with a bounded timeout (ranks that wait for a
    missing peer end with an error instead of hanging)."""
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)


def utterance_for_rank(rank: int, base_seed: int = 7) -> dict:
    """The utterance rank `rank` decodes: its prompt seed and its sampler
    sequence id (so sampled runs draw independent streams per rank)."""
    return {"prompt_seed": base_seed + rank, "seq_id": rank}


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar over all ranks (identity without a group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_rate(world: int, steps: int, units_per_step: int, max_ms: float) -> float:
    """Whole-job throughput: units all ranks processed / the slowest rank's time."""
    return world * steps * units_per_step / (max_ms / 1e3)
