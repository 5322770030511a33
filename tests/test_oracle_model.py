"""Model-level properties of the CPU restatement (restating the tolerances of
the reference's golden tests as self-consistency checks)."""

import numpy as np
import pytest

from tests.conftest import prompt_ids


def _cos(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def test_int_prefill_is_bit_identical_to_pushing(oracle_lib, small_archive_path):
    m = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT, 0)
    ids = prompt_ids(3, 40)
    fed, pushed = oracle_lib.Session(m), oracle_lib.Session(m)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    assert np.array_equal(fed.logits(), pushed.logits())


def test_float_prefill_agrees_with_stepping(oracle_lib, small_archive_path, kats):
    """crates/model/tests/prefill.rs: batched vs stepped cosine > 0.9995, same argmax."""
    m = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_FLOAT, 0)
    ids = prompt_ids(4, 40)
    fed, pushed = oracle_lib.Session(m), oracle_lib.Session(m)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    a, b = fed.logits(), pushed.logits()
    assert _cos(a, b) > kats["prefill_cosine"]
    assert oracle_lib.argmax(a) == oracle_lib.argmax(b)


def test_full_depth_is_the_base_model(oracle_lib, small_archive_path, kats):
    m = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT, 0)
    full = m.with_depth(4)
    a, b = oracle_lib.Session(m), oracle_lib.Session(full)
    a.feed(prompt_ids(5, 12))
    b.feed(prompt_ids(5, 12))
    assert _cos(a.logits(), b.logits()) > kats["full_depth_cosine"]
    assert np.array_equal(a.logits(), b.logits())


def test_depths_outside_the_ladder_are_refused(oracle_lib, small_archive_path):
    m = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT, 0)
    for depth in (1, 5):
        with pytest.raises(oracle_lib.OracleError) as e:
            m.with_depth(depth)
        assert e.value.status == -3
    assert m.with_depth(2).active_layers() == [0, 3]


def test_int_and_float_modes_agree_like_the_reference_documents(oracle_lib, small_archive_path):
    """docs/parity.md:24: the int8 kernel is within ~0.7% rRMS of the float one."""
    ids = prompt_ids(6, 24)
    out = []
    for mode in (oracle_lib.MODE_INT, oracle_lib.MODE_FLOAT):
        s = oracle_lib.Session(oracle_lib.Model.open(small_archive_path, mode, 0))
        s.feed(ids)
        out.append(s.logits())
    assert _cos(out[0], out[1]) > 0.999
    rel = np.sqrt(np.mean((out[0] - out[1]) ** 2) / np.mean(out[1] ** 2))
    assert rel < 0.05


def test_clone_is_independent(oracle_lib, small_archive_path):
    m = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT, 0)
    base = oracle_lib.Session(m)
    base.feed(prompt_ids(8, 10))
    before = base.logits()
    c = base.clone()
    c.push(42)
    assert np.array_equal(base.logits(), before) and len(c) == 11 and len(base) == 10


def test_threads_do_not_change_results(oracle_lib, small_archive_path):
    ids = prompt_ids(9, 20)
    out = []
    for threads in (1, 4):
        s = oracle_lib.Session(oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_FLOAT, threads))
        s.feed(ids)
        out.append(s.logits())
    assert np.array_equal(out[0], out[1])


def test_argmax_and_statistics_follow_the_generator(oracle_lib):
    v = np.array([1.0, 3.0, 3.0, 2.0], dtype=np.float32)
    assert oracle_lib.argmax(v) == 1
    allowed = np.array([1, 0, 1, 1], dtype=np.uint8)
    assert oracle_lib.argmax_allowed(v, allowed) == 2
    assert oracle_lib.argmax_allowed(v, np.zeros(4, dtype=np.uint8)) == -1
    p, m = oracle_lib.allowed_statistics(v, 2, allowed)
    e = np.exp(v.astype(np.float64) - 3.0)
    assert abs(p - e[2] / (e[0] + e[2] + e[3])) < 1e-5 and abs(m - (e[0] + e[2] + e[3]) / e.sum()) < 1e-5


def test_synthetic_archive_is_deterministic(tmp_path):
    from rustyneedle_b200 import synthetic

    g = synthetic.Geometry(num_layers=2, vocab=512, out_vocab=512, max_seq_len=128)
    a = synthetic.write_archive(str(tmp_path / "a.cact"), 3, g)
    b = synthetic.write_archive(str(tmp_path / "b.cact"), 3, g)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_synthetic_archive_resolves_in_the_oracle(oracle_lib, archive_path):
    m = oracle_lib.Model.open(archive_path, oracle_lib.MODE_INT, 1)
    assert (m.vocab, m.d_model, m.num_heads, m.num_kv_heads, m.num_layers, m.head_dim) == (8192, 512, 8, 4, 20, 64)
    info = m.tensor_info(0)
    assert info == dict(kind=3, rows=8192, columns=512, group=128, bits=4)
    assert m.tensor_info(2)["bits"] == 2


def test_raw_product_is_the_archive_product(oracle_lib, archive_path):
    """nbo_product_raw (the product microbenchmark's checker) runs the archive
    path's code: on the embedding's own codes it gives the same bits."""
    from rustyneedle_b200 import synthetic

    packed, levels, norms = synthetic.embedding_raw(seed=0)
    rows, cols = 8192, 512
    model = oracle_lib.Model.open(archive_path, oracle_lib.MODE_INT, 0)
    rng = np.random.default_rng(3)
    for _ in range(2):
        x = rng.standard_normal(cols).astype(np.float32)
        got = oracle_lib.product_raw(oracle_lib.MODE_INT, 4, packed, levels, norms, rows, cols, x)
        want, _ = model.matrix_product(0, x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _features(**kw):
    from rustyneedle_b200 import synthetic

    return synthetic.Geometry(num_layers=4, max_seq_len=256, **kw)


def test_identity_taps_and_an_unreached_window_change_nothing(oracle_lib):
    """Taps (1, 0, 0) reproduce the model without taps bit for bit, and so does a
    window longer than the context; a shorter window changes the result."""
    from rustyneedle_b200 import synthetic

    plain = synthetic.cached_archive(seed=9, geometry=_features())
    identity = synthetic.cached_archive(seed=9, geometry=_features(conv_taps=3, extra={"identity_taps": True}))
    windowed = synthetic.cached_archive(seed=9, geometry=_features(sliding_window=64, global_layers=0b0001))
    ids = prompt_ids(5, 50)

    def logits(path, n):
        s = oracle_lib.Session(oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0))
        s.feed(ids[:n])
        return s.logits()

    assert np.array_equal(logits(plain, 50).view(np.uint32), logits(identity, 50).view(np.uint32))
    assert np.array_equal(logits(plain, 50).view(np.uint32), logits(windowed, 50).view(np.uint32))
    ids = prompt_ids(5, 90)
    assert not np.array_equal(logits(plain, 90), logits(windowed, 90))


def test_taps_and_window_prefill_agree_with_stepping(oracle_lib, kats):
    """The batched convolution (attention.rs:243-276) against the per-token one
    (attention.rs:83-111), in FLOAT mode: cosine > 0.9995, same argmax."""
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=10, geometry=_features(conv_taps=3, sliding_window=24, global_layers=0b1000))
    m = oracle_lib.Model.open(path, oracle_lib.MODE_FLOAT, 0)
    ids = prompt_ids(6, 60)
    fed, pushed = oracle_lib.Session(m), oracle_lib.Session(m)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    a, b = fed.logits(), pushed.logits()
    assert _cos(a, b) > kats["prefill_cosine"]
    assert oracle_lib.argmax(a) == oracle_lib.argmax(b)


def test_engram_with_zero_value_taps_changes_nothing(oracle_lib):
    """Engram value taps of zero add alpha · 0 (session.rs:187-189): the result is
    the model without sites, bit for bit (the site tensors follow every layer's
    draws, so the layers are the same)."""
    from rustyneedle_b200 import synthetic

    plain = synthetic.cached_archive(seed=13, geometry=_features())
    zero = synthetic.cached_archive(seed=13, geometry=_features(engram_sites=(1, 2), engram_slots=256, extra={"zero_engram_taps": True}))
    live = synthetic.cached_archive(seed=13, geometry=_features(engram_sites=(1, 2), engram_slots=256))
    ids = prompt_ids(7, 30)
    out = []
    for path in (plain, zero, live):
        s = oracle_lib.Session(oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0))
        s.feed(ids)
        out.append(s.logits())
    assert np.array_equal(out[0].view(np.uint32), out[1].view(np.uint32))
    assert not np.array_equal(out[0], out[2])


def test_engram_prefill_agrees_with_stepping(oracle_lib, kats):
    """contribute_batch (engram.rs:108-160) against contribute (engram.rs:68-105)
    in FLOAT mode: cosine > 0.9995, same argmax."""
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=14, geometry=_features(conv_taps=2, engram_sites=(0, 3), engram_slots=256))
    m = oracle_lib.Model.open(path, oracle_lib.MODE_FLOAT, 0)
    ids = prompt_ids(8, 50)
    fed, pushed = oracle_lib.Session(m), oracle_lib.Session(m)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    a, b = fed.logits(), pushed.logits()
    assert _cos(a, b) > kats["prefill_cosine"]
    assert oracle_lib.argmax(a) == oracle_lib.argmax(b)


def test_probe_heads_follow_the_reference_tests(oracle_lib, kats):
    """crates/model/tests/prefill.rs: batched vs stepped head_output(2)[0] within
    0.1 (FLOAT mode); INT feeds equal pushes bit for bit; a head that is not in
    the manifest reads None; a shallower depth pools fewer rows."""
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=15, geometry=_features(probe_heads=(2, 3)))
    ids = prompt_ids(9, 45)
    mf = oracle_lib.Model.open(path, oracle_lib.MODE_FLOAT, 0)
    fed, pushed = oracle_lib.Session(mf), oracle_lib.Session(mf)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    assert abs(fed.head_output(2)[0] - pushed.head_output(2)[0]) < kats["prefill_head_tolerance"]
    mi = oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0)
    fed, pushed = oracle_lib.Session(mi), oracle_lib.Session(mi)
    fed.feed(ids)
    for t in ids:
        pushed.push(int(t))
    for code in (2, 3):
        assert np.array_equal(fed.head_output(code), pushed.head_output(code))
        assert np.array_equal(fed.pooled_readout(code), pushed.pooled_readout(code))
    assert fed.head_output(1) is None
    shallow = oracle_lib.Session(mi.with_depth(2))
    shallow.feed(ids)
    assert shallow.head_output(2).shape == fed.head_output(2).shape
    assert not np.array_equal(shallow.head_output(2), fed.head_output(2))


def test_whistle_cross_attention_restatement(oracle_lib):
    """whistle/src/cross.rs: the memory of an encoder output is deterministic,
    the cross hook changes the decoder's result, and without a cross memory
    a Whistle archive decodes as its plain decoder."""
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=18, geometry=_features(text_vocab=8000))
    m = oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0)
    assert oracle_lib.text_vocab(m) == 8000
    enc = np.random.default_rng(1).standard_normal((120, 512)).astype(np.float32)
    a, b = oracle_lib.CrossMemory(m, enc), oracle_lib.CrossMemory(m, enc)
    for layer in range(4):
        for x, y in zip(a.read(layer, 8), b.read(layer, 8)):
            assert np.array_equal(x, y)
    plain, crossed = oracle_lib.Session(m), oracle_lib.Session(m)
    for t in (1, 8003, 40, 41):
        plain.push(t)
        crossed.push_cross(t, a)
    assert not np.array_equal(plain.logits(), crossed.logits())
    decoder = oracle_lib.Model.open(synthetic.cached_archive(seed=18, geometry=_features()), oracle_lib.MODE_INT, 0)
    twin = oracle_lib.Session(decoder)
    for t in (1, 8003, 40, 41):
        twin.push(t)
    assert np.array_equal(plain.logits(), twin.logits())
