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
    """The `count` prompts of `rank`'s shard.

    Lengths are uniform in [low, high] as a stratified draw: one length from
    each of `count` equal strata of the range, drawn once from `seed_base`,
    so every rank holds the same multiset of lengths and caches the same
    number of positions (weak scaling with equal work per GPU; independent
    draws per rank left up to 7 % more KV on one rank than another). Their
    order and the ids (uniform in [id_low, id_high)) are seeded per rank, so
    a rank's shard does not depend on the number of ranks."""
    span = high - low + 1
    offsets = np.random.default_rng(seed_base).random(count)
    lengths = low + np.floor((np.arange(count) + offsets) * span / count).astype(np.int64)
    rng = np.random.default_rng([seed_base, rank])
    lengths = rng.permutation(lengths)
    return [rng.integers(id_low, id_high, int(n)).astype(np.uint32) for n in lengths]


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


def gather_over_ranks(dist, values: list[float], device: str = "cpu") -> list[list[float]]:
    """Every rank's `values` (the same count on each rank), in rank order."""
    if dist is None:
        return [list(values)]
    import torch

    mine = torch.tensor(values, dtype=torch.float64, device=device)
    parts = [torch.zeros_like(mine) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, mine)
    return [[float(x) for x in p.cpu()] for p in parts]


def close_group(dist) -> None:
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


@dataclass
class ShardResult:
    device: int
    tokens: np.ndarray      # [steps][sequences] chosen ids
    logits: np.ndarray      # [sequences][output_vocab] after the last step
    device_ms: float        # device time of the decode steps (CUDA events on the model's stream)


def decode_on_devices(archive: str, shards: list[list[np.ndarray]], devices: list[int], steps: int,
                      depth: int) -> list[ShardResult]:
    """Greedy-decodes shards[i] on devices[i], all GPUs driven from this one
    process with one host thread per GPU (the threading a single Rust host
    serving several GPUs uses: one model, one CUDA stream and one host thread
    per device, no lock shared between them; the reference's process-wide
    spin pool, crates/kernels/src/pool.rs:42-161, has no counterpart).

    Each thread opens its own model on its device, feeds its shard's prompts
    in shared prefill passes and steps them as one batch; the library
    releases the GIL inside every call, so the devices run concurrently. A
    thread's failure is raised here after every thread has finished."""
    import threading

    if len(shards) != len(devices):
        raise ValueError("one shard per device")
    results: list = [None] * len(devices)
    errors: list = []

    def work(i: int) -> None:
        import rustyneedle_b200 as nb

        try:
            shard = shards[i]
            pages = kv_pages_for(shard, steps + 2, depth)
            model = nb.Model.open(archive, device=devices[i], max_sessions=len(shard) + 1, kv_pages=pages)
            if depth != model.config.num_layers:
                model = model.with_depth(depth)
            sessions = [nb.Session(model) for _ in shard]
            nb.feed_many(sessions, shard)
            batch = nb.Batch(model, sessions)
            import torch

            tokens = torch.zeros(steps * len(shard), dtype=torch.int32, device=f"cuda:{devices[i]}")
            torch.cuda.synchronize(devices[i])  # the fill (torch's stream) before the model's stream writes
            ms = batch.run(steps, None, tokens.data_ptr())  # returns after the run's end event
            logits = np.stack([s.logits() for s in sessions])
            results[i] = ShardResult(devices[i], tokens.cpu().numpy().view(np.uint32).reshape(steps, len(shard)),
                                     logits, ms)
            batch.close()
            for s in sessions:
                s.close()
            model.close()
        except BaseException as e:  # reported by the caller's thread
            errors.append((devices[i], e))

    threads = [threading.Thread(target=work, args=(i,), name=f"needle-gpu{d}") for i, d in enumerate(devices)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        device, e = errors[0]
        raise RuntimeError(f"decoding on device {device} failed: {e}") from e
    return results
