"""Data-parallel decoding across the GPUs of one box.

Sequences are independent (each rustyneedle Session owns its whole state,
crates/model/src/session.rs:17-27), so every rank decodes its own shard with
no collective on the data path. The process group only carries the timing
barrier and the max over ranks of the elapsed time. One process per GPU,
launched by torchrun (RANK / LOCAL_RANK / WORLD_SIZE in the environment).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import numpy as np

# A short process-group timeout: ranks that wait on a rank that has gone end
# their next collective with an error instead of hanging.
GROUP_TIMEOUT_S = 120


@dataclass(frozen=True)
class Ranks:
    rank: int
    world: int
    local: int


def ranks_from_env() -> Ranks:
    return Ranks(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                 int(os.environ.get("LOCAL_RANK", "0")))


def shard_prompts(rank: int, count: int, low: int = 128, high: int = 1024, seed_base: int = 1000,
                  id_low: int = 10, id_high: int = 8000) -> list[np.ndarray]:
    """The `count` prompts of `rank`'s shard: lengths uniform in [low, high],
    ids uniform in [id_low, id_high); seeded per rank, so a rank's shard does
    not depend on the number of ranks (weak scaling)."""
    rng = np.random.default_rng(seed_base + rank)
    lengths = rng.integers(low, high + 1, count)
    return [rng.integers(id_low, id_high, n).astype(np.uint32) for n in lengths]


def kv_pages_for(prompts: list[np.ndarray], extra_tokens: int, layers: int, spare_per_layer: int = 40) -> int:
    """64-position pages a shard needs: every prompt plus `extra_tokens`
    decoded tokens, at every layer, plus a spare pool."""
    per_layer = sum(-(-(len(p) + extra_tokens) // 64) for p in prompts)
    return (per_layer + spare_per_layer) * layers


def init_group(ranks: Ranks, backend: str):
    """Initialises the process group (127.0.0.1 rendezvous from torchrun's
    environment); returns the torch.distributed module, or None for one rank."""
    if ranks.world <= 1:
        return None
    import torch
    import torch.distributed as dist

    kwargs = {}
    if backend == "nccl":
        torch.cuda.set_device(ranks.local)
        kwargs["device_id"] = torch.device("cuda", ranks.local)
    dist.init_process_group(backend, timeout=timedelta(seconds=GROUP_TIMEOUT_S), **kwargs)
    return dist


def barrier(dist) -> None:
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, value: float, device: str = "cpu") -> float:
    """The largest `value` over all ranks (the job's time is its slowest rank's)."""
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def close_group(dist) -> None:
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
