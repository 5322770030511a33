"""Parity of the Whistle cross-attention decoder (crates/whistle/src/cross.rs,
lib.rs:240-305) with the CPU restatement in INT mode: the cross memory of an
encoder output bit-exact, and decoding through the cross hook (single
sessions, batches, clones) bit-exact in logits and greedy text tokens. The
archive is a synthetic Whistle: a 4-layer Needle-3 decoder, text vocabulary
8000, and random encoder outputs standing in for the audio encoder."""

import numpy as np
import pytest

from tests.conftest import prompt_ids

pytestmark = pytest.mark.gpu

TEXT_VOCAB = 8000


def _bits_equal(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _mismatch(a, b):
    a, b = np.asarray(a, dtype=np.float32).ravel(), np.asarray(b, dtype=np.float32).ravel()
    bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    return "equal" if bad.size == 0 else f"{bad.size} of {a.size} differ; first at {bad[0]}: {a[bad[0]]!r} vs {b[bad[0]]!r}"


def _text_mask():
    bits = np.zeros(8192, dtype=bool)
    bits[:TEXT_VOCAB] = True
    return np.packbits(bits, bitorder="little").view(np.uint32)


@pytest.fixture(scope="module")
def whistle_path():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=19, geometry=synthetic.Geometry(num_layers=4, max_seq_len=512, text_vocab=TEXT_VOCAB))


@pytest.fixture(scope="module")
def whistle_model(native_built, whistle_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(whistle_path, max_sessions=16)


@pytest.fixture(scope="module")
def whistle_oracle(oracle_lib, whistle_path):
    return oracle_lib.Model.open(whistle_path, oracle_lib.MODE_INT, 0)


def _encoded(seed, frames):
    return np.random.default_rng(seed).standard_normal((frames, 512)).astype(np.float32)


def test_cross_memory_is_bit_exact(whistle_model, whistle_oracle, oracle_lib):
    """CrossWeights::memory over 1500 frames (a 30-second window): every layer's
    keys, values and scales."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug

    assert whistle_model.text_vocab() == TEXT_VOCAB
    enc = _encoded(1, 1500)
    mem = nb.CrossMemory(whistle_model, enc)
    omem = oracle_lib.CrossMemory(whistle_oracle, enc)
    for layer in range(4):
        got, want = debug.cross_memory(mem, layer, 8), omem.read(layer, 8)
        assert np.array_equal(got[0], want[0]) and np.array_equal(got[2], want[2]), layer
        assert _bits_equal(got[1], want[1]) and _bits_equal(got[3], want[3]), layer
    mem.close()


def test_whistle_decode_matches_the_oracle(whistle_model, whistle_oracle, oracle_lib):
    """Whistle::decode's token loop: bos and a language token through the cross
    hook, then greedy steps restricted to the text vocabulary."""
    import rustyneedle_b200 as nb

    enc = _encoded(2, 300)
    mem = nb.CrossMemory(whistle_model, enc)
    omem = oracle_lib.CrossMemory(whistle_oracle, enc)
    s = nb.Session(whistle_model)
    s.set_cross(mem)
    o = oracle_lib.Session(whistle_oracle)
    for t in (1, TEXT_VOCAB + 5):
        s.push(t)
        o.push_cross(t, omem)
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    mask = _text_mask()
    allowed = np.zeros(8192, dtype=np.uint8)
    allowed[:TEXT_VOCAB] = 1
    for _ in range(12):
        token = oracle_lib.argmax_allowed(o.logits(), allowed)
        o.push_cross(token, omem)
        assert s.step(mask) == token
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    # a clone attends to the same memory; a detached session decodes as the plain decoder
    c, oc = s.clone(), o.clone()
    c.push(33)
    oc.push_cross(33, omem)
    assert _bits_equal(c.logits(), oc.logits())
    c.set_cross(None)
    oc2 = o.clone()
    c2 = s.clone()
    c2.set_cross(None)
    c2.push(34)
    oc2.push(34)
    assert _bits_equal(c2.logits(), oc2.logits())
    for x in (s, c, c2):
        x.close()
    mem.close()


@pytest.mark.parametrize("count", [3, 12])
def test_whistle_batched_decode(whistle_model, whistle_oracle, oracle_lib, count):
    """Several sessions, each with its own memory (100 to 700 frames), decoded
    as one batch under the text-vocabulary mask."""
    import rustyneedle_b200 as nb

    mask = np.tile(_text_mask(), count)
    allowed = np.zeros(8192, dtype=np.uint8)
    allowed[:TEXT_VOCAB] = 1
    sessions, oracles, mems, omems = [], [], [], []
    for i in range(count):
        enc = _encoded(100 + i, 100 + 60 * i)
        mems.append(nb.CrossMemory(whistle_model, enc))
        omems.append(oracle_lib.CrossMemory(whistle_oracle, enc))
        s = nb.Session(whistle_model)
        s.set_cross(mems[-1])
        o = oracle_lib.Session(whistle_oracle)
        for t in (1, TEXT_VOCAB + i):
            s.push(t)
            o.push_cross(t, omems[-1])
        sessions.append(s)
        oracles.append(o)
    batch = nb.Batch(whistle_model, sessions)
    for _ in range(4):
        got = batch.step(mask)
        want = []
        for o, om in zip(oracles, omems):
            token = oracle_lib.argmax_allowed(o.logits(), allowed)
            o.push_cross(token, om)
            want.append(token)
        assert list(got) == want
    batch.close()
    for s, o in zip(sessions, oracles):
        assert _bits_equal(s.logits(), o.logits())
        s.close()
    for m in mems:
        m.close()
