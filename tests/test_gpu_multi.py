"""Several GPUs served from one process, one host thread per GPU
(rustyneedle_b200.dp.decode_on_devices), against one GPU.

Sequences share no state (session.rs:17-27), so a sequence's greedy tokens
and final logits may not depend on which GPU decodes it or on which other
sequences share its batch: two shards of config-2-shaped sequences (ranks 0
and 1 of dp.shard_prompts, depth 20) decoded on devices 0 and 1 concurrently
must equal the same sequences decoded together on device 0 alone. Runs where
at least two GPUs are visible."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _device_count() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_two_gpus_one_thread_each_equal_one_gpu(native_built, archive_path):
    from rustyneedle_b200 import dp

    steps, per_shard = 24, 12
    shards = [dp.shard_prompts(rank, per_shard) for rank in (0, 1)]
    split = dp.decode_on_devices(archive_path, shards, [0, 1], steps, depth=20)
    assert [r.device for r in split] == [0, 1]
    (together,) = dp.decode_on_devices(archive_path, [shards[0] + shards[1]], [0], steps, depth=20)
    got = np.concatenate([split[0].tokens, split[1].tokens], axis=1)
    assert np.array_equal(got, together.tokens)
    logits = np.concatenate([split[0].logits, split[1].logits])
    assert np.array_equal(logits.view(np.uint32), together.logits.view(np.uint32))
