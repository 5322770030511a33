"""Failure detection on the GPU without a GPU fault: a bounded device wait that
runs out is reported as NB_ERR_TIMEOUT and leaves the device usable.

nb_debug_expire_waits makes the next routing CTAs give up a short bounded
wait on a barrier that no copy will complete and wait for their own bulk
copies before they leave (so nothing asynchronous outlives them), exactly the path an expired wait of the
token loop takes: the engine's error flag is set, and the next synchronising
call reports the status. Afterwards a fresh session on the same model, and a
fresh model on the same device, decode bit-identically to the CPU
restatement."""

import numpy as np
import pytest

from tests.conftest import prompt_ids

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_an_expired_wait_is_a_timeout_status(native_built, small_archive_path, oracle_lib):
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug

    model = nb.Model.open(small_archive_path, max_sessions=8)
    ids = prompt_ids(31, 20)
    s = nb.Session(model)
    debug.expire_waits(model, 1)
    with pytest.raises(nb.NeedleError) as err:
        s.feed(ids)
    assert err.value.status == -9  # NB_ERR_TIMEOUT
    s.close()

    # the batched step graph reports it too
    a, b = nb.Session(model), nb.Session(model)
    a.feed(ids[:5])
    b.feed(ids[:9])
    batch = nb.Batch(model, [a, b])
    batch.step()
    debug.expire_waits(model, 2)
    with pytest.raises(nb.NeedleError) as err:
        batch.step()
    assert err.value.status == -9
    batch.close()
    a.close()
    b.close()

    omodel = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT, 0)
    o = oracle_lib.Session(omodel)
    o.feed(ids)
    want = o.logits()
    # the same model, a fresh session
    fresh = nb.Session(model)
    fresh.feed(ids)
    assert _bits_equal(fresh.logits(), want)
    fresh.close()
    # a fresh model on the same device
    other = nb.Model.open(small_archive_path, max_sessions=2)
    t = nb.Session(other)
    t.feed(ids)
    assert _bits_equal(t.logits(), want)
    t.close()
    other.close()
    model.close()
