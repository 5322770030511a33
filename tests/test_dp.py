"""The multi-rank host path (rustyneedle_b200.dp) on CPU with two gloo ranks:
shards are disjoint and independent of the world size, the timing reduction
takes the slowest rank, and decoding each rank's shard separately gives the
same tokens as decoding every sequence in one process (sequences share no
state; the CPU restatement stands in for the device here)."""

import os
import socket

import numpy as np
import pytest

from rustyneedle_b200 import dp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(oracle, archive, prompts, steps):
    model = oracle.Model.open(archive, oracle.MODE_INT, 1)
    out = []
    for ids in prompts:
        s = oracle.Session(model)
        s.feed(ids)
        tokens = []
        for _ in range(steps):
            t = oracle.argmax(s.logits())
            tokens.append(t)
            s.push(t)
        out.append(tokens)
    return np.array(out, dtype=np.uint32)


def _rank_main(rank, world, port, archive, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oracle import oracle

    ranks = dp.ranks_from_env()
    dist = dp.init_group(ranks, "gloo")
    shard = [p[:6] for p in dp.shard_prompts(ranks.rank, 3, 8, 12)]
    tokens = _decode(oracle, archive, shard, steps=2)
    dp.barrier(dist)
    slowest = dp.max_over_ranks(dist, float(10 + ranks.rank))
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), tokens=tokens, slowest=slowest,
             lengths=np.array([len(p) for p in dp.shard_prompts(ranks.rank, 3, 8, 12)]))
    dp.close_group(dist)


def test_shards_are_seeded_per_rank_and_disjoint():
    a0 = dp.shard_prompts(0, 4)
    a1 = dp.shard_prompts(1, 4)
    assert all(np.array_equal(x, y) for x, y in zip(a0, dp.shard_prompts(0, 4)))
    assert not any(len(x) == len(y) and np.array_equal(x, y) for x in a0 for y in a1)
    assert all(128 <= len(p) <= 1024 for p in a0 + a1)
    assert dp.kv_pages_for([np.zeros(64), np.zeros(65)], 0, 2, spare_per_layer=1) == (1 + 2 + 1) * 2


def test_two_gloo_ranks_decode_their_shards_like_one_process(oracle_lib, small_archive_path, tmp_path):
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    mp.start_processes(_rank_main, args=(world, port, small_archive_path, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    results = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    assert all(float(r["slowest"]) == 11.0 for r in results)
    together = [p[:6] for r in range(world) for p in dp.shard_prompts(r, 3, 8, 12)]
    want = _decode(oracle_lib, small_archive_path, together, steps=2)
    got = np.concatenate([r["tokens"] for r in results])
    assert np.array_equal(got, want)


def test_one_rank_needs_no_group():
    assert dp.init_group(dp.Ranks(0, 1, 0), "gloo") is None
    assert dp.max_over_ranks(None, 3.5) == 3.5
    dp.barrier(None)
    dp.close_group(None)


def test_decode_on_devices_reports_a_thread_failure(native_built, archive_path):
    """A device thread that fails (here: no GPU, or a device ordinal that does
    not exist) is reported to the caller after every thread has finished."""
    shards = [dp.shard_prompts(0, 1, 8, 12), dp.shard_prompts(1, 1, 8, 12)]
    with pytest.raises(RuntimeError, match="decoding on device"):
        dp.decode_on_devices(archive_path, shards, [999, 998], 1, depth=2)
    with pytest.raises(ValueError):
        dp.decode_on_devices(archive_path, shards, [0], 1, depth=2)


def test_gather_over_one_rank():
    assert dp.gather_over_ranks(None, [1.5, 2.0]) == [[1.5, 2.0]]
