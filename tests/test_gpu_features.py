"""Parity of the archive features the default synthetic geometry leaves out:
QKV causal convolution taps (model/src/attention.rs:83-117, 243-276), the
sliding window with global layers (attention.rs:171-177), engram sites
(model/src/engram.rs, session.rs:93-113, 180-190) and probe heads
(model/src/heads.rs, session.rs:144-160). The archives are 6-layer
synthetic models with 3 taps, a 40-position window and layers 0 and 5
global, with engram sites and probe heads added in the later groups; every
case is bit-exact against the CPU restatement in INT mode."""

import numpy as np
import pytest

from tests.conftest import prompt_ids

pytestmark = pytest.mark.gpu

WINDOW = 40


def _bits_equal(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _mismatch(a, b):
    a, b = np.asarray(a, dtype=np.float32).ravel(), np.asarray(b, dtype=np.float32).ravel()
    bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    if bad.size == 0:
        return "equal"
    i = bad[0]
    return f"{bad.size} of {a.size} differ; first at {i}: {a[i]!r} vs {b[i]!r}"


def _geometry(taps: int = 3):
    from rustyneedle_b200 import synthetic

    return synthetic.Geometry(num_layers=6, max_seq_len=512, conv_taps=taps, sliding_window=WINDOW, global_layers=0b100001)


@pytest.fixture(scope="module")
def features_path():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=7, geometry=_geometry())


@pytest.fixture(scope="module")
def features_model(native_built, features_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(features_path, max_sessions=96)


@pytest.fixture(scope="module")
def features_oracle(oracle_lib, features_path):
    return oracle_lib.Model.open(features_path, oracle_lib.MODE_INT, 0)


def test_windowed_prefill_matches_hidden_logits_and_cache(features_model, features_oracle, oracle_lib):
    """One 150-token pass: every position past the first mixes same-pass rows;
    the windowed layers attend to their last 40 positions only."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug

    ids = prompt_ids(31, 150)
    s = nb.Session(features_model)
    s.feed(ids)
    o = oracle_lib.Session(features_oracle)
    o.feed(ids)
    for layer in features_model.active_layers():
        keys, ks, values, vs = debug.kv(s, layer)
        okeys, oks, ovalues, ovs = o.cache(layer)
        assert np.array_equal(keys, okeys) and np.array_equal(values, ovalues), layer
        assert _bits_equal(ks, oks) and _bits_equal(vs, ovs), layer
    assert _bits_equal(debug.hidden(s), o.hidden()), _mismatch(debug.hidden(s), o.hidden())
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    s.close()


def test_ragged_feeds_then_greedy_steps(features_model, features_oracle, oracle_lib):
    """Feeds of 1, 2, 5, 64, 1 and 3 tokens (the convolution reads across every
    pass boundary, from the ring), then 12 greedy steps past the window."""
    import rustyneedle_b200 as nb

    s = nb.Session(features_model)
    o = oracle_lib.Session(features_oracle)
    at = 0
    ids = prompt_ids(32, 76)
    for n in (1, 2, 5, 64, 1, 3):
        s.feed(ids[at:at + n])
        o.feed(ids[at:at + n])
        at += n
        assert _bits_equal(s.logits(), o.logits()), (at, _mismatch(s.logits(), o.logits()))
    for _ in range(12):
        token = oracle_lib.argmax(o.logits())
        o.push(token)
        assert s.step() == token
    assert _bits_equal(s.logits(), o.logits())
    s.close()


def test_small_passes_split_a_prompt_anywhere(native_built, features_path, features_oracle, oracle_lib):
    """max_batch_tokens 7: a 90-token prompt runs as 13 passes, so the taps of
    the first rows of every pass come from the previous pass's ring rows."""
    import rustyneedle_b200 as nb

    model = nb.Model.open(features_path, max_sessions=4, max_batch_tokens=7)
    ids = prompt_ids(33, 90)
    s = nb.Session(model)
    s.feed(ids)
    o = oracle_lib.Session(features_oracle)
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    s.close()
    model.close()


@pytest.mark.parametrize("count", [6, 72])
def test_batched_decode_with_taps_and_window(features_model, features_oracle, oracle_lib, count):
    """Batched steps (6 sequences: cluster kernels; 72: one CTA per token), some
    sequences shorter than the taps, with a clone forked mid-way."""
    import rustyneedle_b200 as nb

    base = [1, 2, 3, 39, 41, 120]
    lengths = (base * (count // len(base) + 1))[:count]
    sessions, oracles = [], []
    for i, n in enumerate(lengths):
        ids = prompt_ids(700 + i, n)
        s = nb.Session(features_model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(features_oracle)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(features_model, sessions)
    for _ in range(3):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    batch.close()
    # a clone carries the convolution history with it
    c, oc = sessions[4].clone(), oracles[4].clone()
    sessions[4].push(17)
    oracles[4].push(17)
    c.push(18)
    oc.push(18)
    assert _bits_equal(sessions[4].logits(), oracles[4].logits())
    assert _bits_equal(c.logits(), oc.logits()), _mismatch(c.logits(), oc.logits())
    for s in sessions + [c]:
        s.close()


@pytest.mark.parametrize("taps", [1, 2])
def test_short_tap_counts(native_built, oracle_lib, taps):
    """One tap (no history) and two taps (a one-row ring)."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=8, geometry=_geometry(taps))
    model = nb.Model.open(path, max_sessions=4)
    omodel = oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0)
    s = nb.Session(model)
    o = oracle_lib.Session(omodel)
    ids = prompt_ids(34, 50)
    s.feed(ids[:45])
    o.feed(ids[:45])
    for t in ids[45:]:
        s.push(int(t))
        o.push(int(t))
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    s.close()
    model.close()


# ------------------------------------------------------------- engram sites
def _engram_geometry(**kw):
    from rustyneedle_b200 import synthetic

    base = dict(num_layers=6, max_seq_len=512, conv_taps=3, sliding_window=WINDOW, global_layers=0b100001, engram_sites=(1, 4),
                engram_slots=512, engram_orders=(2, 3), engram_heads_per_order=2, engram_conv_taps=3, engram_dilation=2)
    base.update(kw)
    return synthetic.Geometry(**base)


@pytest.fixture(scope="module")
def engram_path():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=11, geometry=_engram_geometry())


@pytest.fixture(scope="module")
def engram_model(native_built, engram_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(engram_path, max_sessions=96)


@pytest.fixture(scope="module")
def engram_oracle(oracle_lib, engram_path):
    return oracle_lib.Model.open(engram_path, oracle_lib.MODE_INT, 0)


def test_engram_prefill_and_ragged_feeds(engram_model, engram_oracle, oracle_lib):
    """Two engram sites (orders 2 and 3, value taps 3 at dilation 2) with the
    QKV taps and the window: one 100-token pass, then ragged feeds whose hashes
    and value taps read across pass boundaries, then greedy steps."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug

    ids = prompt_ids(41, 100)
    s = nb.Session(engram_model)
    s.feed(ids)
    o = oracle_lib.Session(engram_oracle)
    o.feed(ids)
    assert _bits_equal(debug.hidden(s), o.hidden()), _mismatch(debug.hidden(s), o.hidden())
    more = prompt_ids(42, 40)
    at = 0
    for n in (1, 2, 5, 30, 1, 1):
        s.feed(more[at:at + n])
        o.feed(more[at:at + n])
        at += n
        assert _bits_equal(s.logits(), o.logits()), (at, _mismatch(s.logits(), o.logits()))
    for _ in range(10):
        token = oracle_lib.argmax(o.logits())
        o.push(token)
        assert s.step() == token
    s.close()


def test_engram_small_passes_and_clone(native_built, engram_path, engram_oracle, oracle_lib):
    """max_batch_tokens 5: the token and value rings carry every pass boundary;
    a clone carries both rings."""
    import rustyneedle_b200 as nb

    model = nb.Model.open(engram_path, max_sessions=4, max_batch_tokens=5)
    ids = prompt_ids(43, 61)
    s = nb.Session(model)
    s.feed(ids)
    o = oracle_lib.Session(engram_oracle)
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    c, oc = s.clone(), o.clone()
    for t in (5, 6, 7):
        c.push(t)
        oc.push(t)
    s.push(9)
    o.push(9)
    assert _bits_equal(c.logits(), oc.logits()) and _bits_equal(s.logits(), o.logits())
    for x in (s, c):
        x.close()
    model.close()


@pytest.mark.parametrize("count", [6, 72])
def test_engram_batched_decode(engram_model, engram_oracle, oracle_lib, count):
    import rustyneedle_b200 as nb

    base = [1, 2, 3, 5, 8, 60]
    lengths = (base * (count // len(base) + 1))[:count]
    sessions, oracles = [], []
    for i, n in enumerate(lengths):
        ids = prompt_ids(800 + i, n)
        s = nb.Session(engram_model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(engram_oracle)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(engram_model, sessions)
    for _ in range(4):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    batch.close()
    for s, o in zip(sessions, oracles):
        assert _bits_equal(s.logits(), o.logits())
        s.close()


def test_engram_depth_without_a_site(engram_model, engram_oracle, oracle_lib):
    """Depth 5 (layers 0, 1, 2, 3, 5) keeps the site on layer 1 and skips the one
    on layer 4: that site neither contributes nor keeps history."""
    import rustyneedle_b200 as nb

    model, omodel = engram_model.with_depth(5), engram_oracle.with_depth(5)
    assert model.active_layers() == [0, 1, 2, 3, 5]
    ids = prompt_ids(44, 70)
    s = nb.Session(model)
    s.feed(ids)
    o = oracle_lib.Session(omodel)
    o.feed(ids)
    s.push(3)
    o.push(3)
    assert _bits_equal(s.logits(), o.logits()), (model.active_layers(), _mismatch(s.logits(), o.logits()))
    s.close()


@pytest.mark.parametrize("variant", ["k256", "k2048_seed", "dilation1_taps1"])
def test_engram_variants(native_built, oracle_lib, variant):
    """Tables x sub_dim 256 (padded to a 512 product), 1024 (padded to 2048,
    four orders, seed heads 3, stepped as a 256-sequence batch: two step
    groups), and one value tap (no ring)."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import synthetic

    kw = {"k256": dict(engram_orders=(2,), engram_heads_per_order=2, engram_sites=(2,)),
          "k2048_seed": dict(engram_orders=(1, 2, 3, 4), engram_heads_per_order=2, engram_seed_heads=3, engram_sites=(0, 3, 5)),
          "dilation1_taps1": dict(engram_conv_taps=1, engram_dilation=1)}[variant]
    path = synthetic.cached_archive(seed=12, geometry=_engram_geometry(**kw))
    sequences = 256 if variant == "k2048_seed" else 4
    model = nb.Model.open(path, max_sessions=sequences)
    omodel = oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0)
    sessions, oracles = [], []
    for i in range(sequences):
        ids = prompt_ids(900 + i, 1 + i % 7 if sequences > 4 else 30 + i)
        s = nb.Session(model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(omodel)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(model, sessions)
    for _ in range(2):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    batch.close()
    for s, o in zip(sessions, oracles):
        assert _bits_equal(s.logits(), o.logits())
        s.close()
    model.close()


# -------------------------------------------------------------- probe heads
def _heads_geometry(**kw):
    base = dict(probe_heads=(2, 3), probes_per_layer=2, head_queries=2, head_outputs=3)
    base.update(kw)
    return _engram_geometry(**base)


@pytest.fixture(scope="module")
def heads_path():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=16, geometry=_heads_geometry())


@pytest.fixture(scope="module")
def heads_model(native_built, heads_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(heads_path, max_sessions=96)


@pytest.fixture(scope="module")
def heads_oracle(oracle_lib, heads_path):
    return oracle_lib.Model.open(heads_path, oracle_lib.MODE_INT, 0)


def _heads_equal(s, o):
    for code in (2, 3):
        got, want = s.head_output(code), o.head_output(code)
        assert _bits_equal(got, want), (code, _mismatch(got, want))
        got, want = s.pooled_readout(code), o.pooled_readout(code)
        assert _bits_equal(got, want), (code, _mismatch(got, want))
    assert s.head_output(1) is None and o.head_output(1) is None


def test_heads_after_prefill_ragged_feeds_and_steps(heads_model, heads_oracle, oracle_lib):
    """ProbeHead::observe over a 90-token pass (one run: the online softmax in
    position order), ragged feeds and greedy steps; head_output and
    pooled_readout of heads 2 and 3 (code 3 carries a calibration tensor)."""
    import rustyneedle_b200 as nb

    s = nb.Session(heads_model)
    o = oracle_lib.Session(heads_oracle)
    ids = prompt_ids(51, 90)
    s.feed(ids)
    o.feed(ids)
    _heads_equal(s, o)
    more = prompt_ids(52, 12)
    at = 0
    for n in (1, 3, 7, 1):
        s.feed(more[at:at + n])
        o.feed(more[at:at + n])
        at += n
    for _ in range(5):
        token = oracle_lib.argmax(o.logits())
        o.push(token)
        assert s.step() == token
    _heads_equal(s, o)
    c, oc = s.clone(), o.clone()
    c.push(21)
    oc.push(21)
    _heads_equal(c, oc)
    _heads_equal(s, o)
    s.close()
    c.close()


def test_heads_over_small_passes_and_a_shallow_depth(native_built, heads_path, heads_oracle, oracle_lib):
    """max_batch_tokens 5 splits one prompt over many passes (each a run of its
    own); depth 3 pools the embedding cell and its three layers only."""
    import rustyneedle_b200 as nb

    model = nb.Model.open(heads_path, max_sessions=4, max_batch_tokens=5)
    ids = prompt_ids(53, 47)
    for depth in (6, 3):
        m = model if depth == 6 else model.with_depth(depth)
        om = heads_oracle if depth == 6 else heads_oracle.with_depth(depth)
        s = nb.Session(m)
        s.feed(ids)
        o = oracle_lib.Session(om)
        o.feed(ids)
        _heads_equal(s, o)
        s.close()
    model.close()


@pytest.mark.parametrize("count", [6, 72])
def test_heads_after_batched_decode(heads_model, heads_oracle, oracle_lib, count):
    import rustyneedle_b200 as nb

    base = [1, 4, 9, 30]
    lengths = (base * (count // len(base) + 1))[:count]
    sessions, oracles = [], []
    for i, n in enumerate(lengths):
        ids = prompt_ids(1000 + i, n)
        s = nb.Session(heads_model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(heads_oracle)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(heads_model, sessions)
    for _ in range(3):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    batch.close()
    for s, o in list(zip(sessions, oracles))[:8]:
        _heads_equal(s, o)
    for s in sessions:
        s.close()


def test_one_query_head_projects_through_a_512_product(native_built, oracle_lib):
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=17, geometry=_heads_geometry(probe_heads=(2, 3, 1), head_queries=1, probes_per_layer=3,
                                                                      engram_sites=()))
    model = nb.Model.open(path, max_sessions=2)
    omodel = oracle_lib.Model.open(path, oracle_lib.MODE_INT, 0)
    s, o = nb.Session(model), oracle_lib.Session(omodel)
    ids = prompt_ids(54, 33)
    s.feed(ids)
    o.feed(ids)
    for code in (1, 2, 3):
        assert _bits_equal(s.head_output(code), o.head_output(code)), code
    s.close()
    model.close()
