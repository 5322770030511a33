"""Parity of the sm_100a path with the CPU restatement (INT mode = the
reference's integer kernels), called through the C ABI.

The bar: integer work bit-exact; every float the reference fixes the order of
(hidden states, logits, KV scales) bit-exact as well, so greedy tokens are
identical. The sequential-sum statistics use the reference's order too and
are held to 1e-6 relative."""

import ctypes

import numpy as np
import pytest

from tests.conftest import prompt_ids, random_mask

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def device_model(native_built, archive_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(archive_path, max_sessions=64)


@pytest.fixture(scope="module")
def oracle_model(oracle_lib, archive_path):
    return oracle_lib.Model.open(archive_path, oracle_lib.MODE_INT, 0)


def _bits_equal(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _mismatch(a, b):
    a, b = np.asarray(a, dtype=np.float32).ravel(), np.asarray(b, dtype=np.float32).ravel()
    bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    if bad.size == 0:
        return "equal"
    i = bad[0]
    rel = np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30))
    return f"{bad.size} of {a.size} differ; first at {i}: {a[i]!r} vs {b[i]!r}; max rel {rel:.3g}"


# ------------------------------------------------------------------ kernels
def test_device_exponential_reproduces_host_libm(device_model):
    from rustyneedle_b200 import debug

    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-110, 89, 200_000), rng.standard_normal(200_000) * 4,
                        [0.0, -0.0, 88.7, 88.73, 89.0, -103.9, -104.0, -110.0, 1e-30, -1e-30]]).astype(np.float32)
    # inputs the libm rounds differently from the correctly rounded result
    table = np.fromfile(__import__("rustyneedle_b200.build", fromlist=["x"]).EXPF_TABLE, dtype=np.uint32)[3:]
    listed = table[rng.integers(0, table.size, 20_000)].view(np.float32)
    x = np.concatenate([x, listed])
    want = np.array([libm.expf(float(v)) for v in x], dtype=np.float32)
    got = debug.math(device_model, debug.OP_EXPF, x)
    assert _bits_equal(got, want), _mismatch(got, want)


def test_device_sigmoid_fast_exp_silu_match_the_oracle(device_model, oracle_lib):
    from rustyneedle_b200 import debug

    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(50_000) * 6, rng.uniform(-100, 100, 20_000)]).astype(np.float32)
    sig = np.array([oracle_lib.sigmoid(v) for v in x], dtype=np.float32)
    assert _bits_equal(debug.math(device_model, debug.OP_SIGMOID, x), sig)
    fe = np.array([oracle_lib.fast_exp(v) for v in x], dtype=np.float32)
    assert _bits_equal(debug.math(device_model, debug.OP_FAST_EXP, x), fe)


def test_sinkhorn_reciprocal_is_correctly_rounded(device_model):
    """The Sinkhorn's 1 / max(total, f32::MIN_POSITIVE) (ops.rs:206, 211) over every
    64th binary32 in [2^-126, 4] plus zeros, negatives and NaN (-> MIN_POSITIVE);
    numpy's float32 division is the IEEE correctly rounded quotient."""
    from rustyneedle_b200 import debug

    bits = np.arange(0x00800000, 0x40800001, 64, dtype=np.uint32)
    x = np.concatenate([bits.view(np.float32), np.array([0.0, -0.0, -1.0, np.nan, 4.0], dtype=np.float32)])
    want = (np.float32(1.0) / np.maximum(np.nan_to_num(x, nan=0.0), np.finfo(np.float32).tiny)).astype(np.float32)
    got = debug.math(device_model, debug.OP_SINKHORN_RCP, x)
    assert _bits_equal(got, want), _mismatch(got, want)


def _tensor_index(oracle_model, want):
    """Archive index of a tensor by its canonical position (layout.rs:190-230)."""
    layers, per_layer = oracle_model.num_layers, 24
    name, layer = want
    offsets = {"q": 2, "k": 3, "v": 4, "gate": 7, "out": 8}
    if name == "embedding":
        return 0
    return 1 + layer * per_layer + offsets[name] - 1


@pytest.mark.parametrize("layer", [0, 7, 19])
def test_fused_projection_matches_the_panel_kernel(device_model, oracle_model, layer):
    from rustyneedle_b200 import debug

    rng = np.random.default_rng(layer)
    x = (rng.standard_normal((5, 512)) * rng.uniform(0.01, 3.0, (5, 1))).astype(np.float32)
    x[4, :] = 0.0  # an all-zero input: every group scale falls back to 1
    got = debug.project(device_model, debug.MATRIX_QKVG, layer, x, 1536)
    start = 0
    for name, rows in (("q", 512), ("k", 256), ("v", 256), ("gate", 512)):
        tensor = _tensor_index(oracle_model, (name, layer))
        for t in range(x.shape[0]):
            want, _ = oracle_model.matrix_product(tensor, x[t])
            assert _bits_equal(got[t, start:start + rows], want), (name, t, _mismatch(got[t, start:start + rows], want))
        start += rows


@pytest.mark.parametrize("tokens", [17, 40, 300])
def test_projection_over_many_token_tiles(device_model, oracle_model, tokens):
    from rustyneedle_b200 import debug

    rng = np.random.default_rng(tokens)
    x = (rng.standard_normal((tokens, 512)) * rng.uniform(0.01, 3.0, (tokens, 1))).astype(np.float32)
    got = debug.project(device_model, debug.MATRIX_QKVG, 4, x, 1536)
    start = 0
    for name, rows in (("q", 512), ("k", 256), ("v", 256), ("gate", 512)):
        tensor = _tensor_index(oracle_model, (name, 4))
        for t in range(0, tokens, 7):
            want, _ = oracle_model.matrix_product(tensor, x[t])
            assert _bits_equal(got[t, start:start + rows], want), (name, t, _mismatch(got[t, start:start + rows], want))
        start += rows


@pytest.mark.parametrize("layer", [0, 11])
def test_hadamard_mlp_matches(device_model, oracle_model, layer):
    from rustyneedle_b200 import debug

    rng = np.random.default_rng(50 + layer)
    x = rng.standard_normal((6, 512)).astype(np.float32)
    got = debug.hadamard(device_model, layer, x)
    for t in range(6):
        want = oracle_model.hadamard(layer, x[t])
        assert _bits_equal(got[t], want), (t, _mismatch(got[t], want))


def test_out_projection_and_logit_rows_match(device_model, oracle_model):
    from rustyneedle_b200 import debug

    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    got = debug.project(device_model, debug.MATRIX_OUT, 3, x, 512)
    tensor = _tensor_index(oracle_model, ("out", 3))
    for t in range(3):
        want, _ = oracle_model.matrix_product(tensor, x[t])
        assert _bits_equal(got[t], want), _mismatch(got[t], want)
    got = debug.project(device_model, debug.MATRIX_LOGITS, 0, x, 8192)
    for t in range(3):
        want, _ = oracle_model.matrix_product(0, x[t])
        assert _bits_equal(got[t], want), _mismatch(got[t], want)


# ------------------------------------------------------------------- model
def test_feed_matches_the_oracle_hidden_logits_and_cache(device_model, oracle_model, oracle_lib):
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug

    model = device_model.with_depth(2)
    omodel = oracle_model.with_depth(2)
    ids = prompt_ids(0, 32)
    s = nb.Session(model)
    s.feed(ids)
    o = oracle_lib.Session(omodel)
    o.feed(ids)
    assert len(s) == len(o) == 32
    for layer in model.active_layers():
        keys, ks, values, vs = debug.kv(s, layer)
        okeys, oks, ovalues, ovs = o.cache(layer)
        assert np.array_equal(keys, okeys) and np.array_equal(values, ovalues), layer
        assert _bits_equal(ks, oks) and _bits_equal(vs, ovs), layer
    assert _bits_equal(debug.hidden(s), o.hidden()), _mismatch(debug.hidden(s), o.hidden())
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())


def test_device_matches_the_numpy_restatement(native_built, small_archive_path):
    """The device against the second, numpy restatement (oracle/restated.py)
    directly: a 4-layer archive, six pushed tokens with the logits after each,
    then four greedy tokens chosen by the device's batch step."""
    import rustyneedle_b200 as nb
    from oracle import restated

    model = nb.Model.open(small_archive_path, max_sessions=2)
    s = nb.Session(model)
    r = restated.Session(restated.Archive(small_archive_path))
    for token in [17, 300, 5000, 42, 9, 1234]:
        s.push(token)
        r.push(token)
        assert _bits_equal(s.logits(), r.logits()), _mismatch(s.logits(), r.logits())
    batch = nb.Batch(model, [s])
    for _ in range(4):
        want = int(np.argmax(r.logits()))  # the first index of the maximum (generator.rs:147-152)
        assert int(batch.step()[0]) == want
        r.push(want)
    batch.close()
    assert _bits_equal(s.logits(), r.logits())
    s.close()
    model.close()


def test_device_features_match_the_numpy_restatement(native_built):
    """The same on an archive with every feature (3-tap q/k/v convolutions,
    a 40-position window on the non-global layers, engram sites at layers 1
    and 4, probe heads 2 and 3): a 12-token feed, then eight pushes, with the
    logits and both heads' outputs after each push."""
    import rustyneedle_b200 as nb
    from oracle import restated
    from rustyneedle_b200 import synthetic

    geometry = synthetic.Geometry(num_layers=6, max_seq_len=512, conv_taps=3, sliding_window=40, global_layers=0b100001,
                                  engram_sites=(1, 4), engram_slots=512, engram_orders=(2, 3), engram_heads_per_order=2,
                                  engram_conv_taps=3, engram_dilation=2, probe_heads=(2, 3), probes_per_layer=2, head_queries=2,
                                  head_outputs=3)
    path = synthetic.cached_archive(seed=16, geometry=geometry)
    model = nb.Model.open(path, max_sessions=2)
    s = nb.Session(model)
    r = restated.Session(restated.Archive(path))
    tokens = [int(t) for t in np.random.default_rng(8).integers(10, 8000, 20)]
    s.feed(tokens[:12])
    for t in tokens[:12]:
        r.push(t)
    assert _bits_equal(s.logits(), r.logits()), _mismatch(s.logits(), r.logits())
    for t in tokens[12:]:
        s.push(t)
        r.push(t)
        assert _bits_equal(s.logits(), r.logits()), _mismatch(s.logits(), r.logits())
        for code in (2, 3):
            assert _bits_equal(s.head_output(code), r.head_output(code)), code
    s.close()
    model.close()


def test_a_shorter_model_opened_later_leaves_the_first_working(archive_path, oracle_model, oracle_lib):
    """Models of different context lengths in one process: the kernels'
    shared-memory limits are per-process function attributes, so opening a
    512-position model after a 2048-position one must not shrink what the
    first one's attention launches take."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import synthetic

    long_model = nb.Model.open(archive_path, max_sessions=2).with_depth(2)
    short_model = nb.Model.open(synthetic.cached_archive(seed=19, geometry=synthetic.Geometry(num_layers=4, max_seq_len=512)),
                                max_sessions=2)
    ids = prompt_ids(13, 1500)
    s = nb.Session(long_model)
    s.feed(ids)
    o = oracle_lib.Session(oracle_model.with_depth(2))
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    short = nb.Session(short_model)
    short.feed(ids[:100])
    s.close()
    short.close()
    short_model.close()
    long_model.close()


def test_long_prefill_matches_the_oracle(device_model, oracle_model, oracle_lib):
    """A 600-token prompt in one pass (19 token blocks of the tcgen05 product, the last ragged)."""
    import rustyneedle_b200 as nb

    ids = prompt_ids(11, 600)
    s = nb.Session(device_model.with_depth(2))
    s.feed(ids)
    o = oracle_lib.Session(oracle_model.with_depth(2))
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits()), _mismatch(s.logits(), o.logits())
    s.close()


def test_config0_greedy_tokens_are_identical(device_model, oracle_model, oracle_lib):
    """Config 0: depth 2, 32 prompt ids, 64 greedy tokens, batch 1, unconstrained."""
    import rustyneedle_b200 as nb

    model = device_model.with_depth(2)
    omodel = oracle_model.with_depth(2)
    ids = prompt_ids(0, 32)
    s = nb.Session(model)
    s.feed(ids)
    o = oracle_lib.Session(omodel)
    o.feed(ids)
    got, want = [], []
    for _ in range(64):
        got.append(s.step())
        token = oracle_lib.argmax(o.logits())
        o.push(token)
        want.append(token)
    assert got == want
    assert _bits_equal(s.logits(), o.logits())


def test_depth20_masked_steps_and_statistics(device_model, oracle_model, oracle_lib):
    """Config-1 style: full depth, a grammar bitset (~5% allowed) every step."""
    import rustyneedle_b200 as nb

    ids = prompt_ids(5, 48)
    s = nb.Session(device_model)
    s.feed(ids)
    o = oracle_lib.Session(oracle_model)
    o.feed(ids)
    rng = np.random.default_rng(9)
    for step in range(12):
        bits, allowed = random_mask(rng, 8192, 0.05)
        token, stats = s.step(bits, stats=True)
        logits = o.logits()
        want = oracle_lib.argmax_allowed(logits, allowed)
        assert token == want, step
        p, m = oracle_lib.allowed_statistics(logits, want, allowed)
        assert abs(stats.probability - p) <= 1e-6 * abs(p) and abs(stats.mass - m) <= 1e-6 * abs(m)
        o.push(want)
    assert _bits_equal(s.logits(), o.logits())


def test_empty_mask_falls_back_to_the_unrestricted_argmax(device_model, oracle_model, oracle_lib):
    import rustyneedle_b200 as nb

    model = device_model.with_depth(2)
    s = nb.Session(model)
    s.feed(prompt_ids(2, 8))
    o = oracle_lib.Session(oracle_model.with_depth(2))
    o.feed(prompt_ids(2, 8))
    token = s.step(np.zeros(8192 // 32, dtype=np.uint32))
    assert token == oracle_lib.argmax(o.logits())


def test_batched_decode_matches_single_sessions(device_model, oracle_model, oracle_lib):
    import rustyneedle_b200 as nb

    model = device_model.with_depth(4)
    omodel = oracle_model.with_depth(4)
    lengths = [3, 17, 64, 65, 130]
    sessions, oracles = [], []
    for i, n in enumerate(lengths):
        ids = prompt_ids(100 + i, n)
        s = nb.Session(model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(omodel)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(model, sessions)
    for _ in range(6):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    for s, o in zip(sessions, oracles):
        assert _bits_equal(s.logits(), o.logits())


def test_feeding_many_sessions_at_once_matches_feeding_each(device_model):
    """nb_sessions_feed packs several prompts into shared passes (one prompt
    spans a pass boundary): every session ends bit-identical to feeding it alone."""
    import rustyneedle_b200 as nb

    model = device_model.with_depth(3)
    lengths = [40, 700, 1, 300, 90]  # 1131 tokens: two passes of up to 1024
    prompts = [prompt_ids(900 + i, n) for i, n in enumerate(lengths)]
    together = [nb.Session(model) for _ in lengths]
    nb.feed_many(together, prompts)
    for s, ids in zip(together, prompts):
        alone = nb.Session(model)
        alone.feed(ids)
        assert len(s) == len(alone) == len(ids)
        assert _bits_equal(s.logits(), alone.logits()), _mismatch(s.logits(), alone.logits())
        alone.close()
    # both continue alike
    a, b = together[1], nb.Session(model)
    b.feed(prompts[1])
    a.push(7)
    b.push(7)
    assert _bits_equal(a.logits(), b.logits())
    for s in together + [b]:
        s.close()


def test_wide_batch_decode_matches_the_oracle(archive_path, oracle_model, oracle_lib):
    """A decode step over more than 64 sequences: the attention does the head step
    itself and prepares the out projection in its last CTA per token, the block
    finish runs one CTA per token, the products run on the tensor cores."""
    import rustyneedle_b200 as nb

    model = nb.Model.open(archive_path, max_sessions=80).with_depth(4)
    omodel = oracle_model.with_depth(4)
    lengths = [5, 33, 64, 97, 130, 190] * 12  # 72 sequences
    sessions, oracles = [], []
    for i, n in enumerate(lengths):
        ids = prompt_ids(500 + i, n)
        s = nb.Session(model)
        s.feed(ids)
        sessions.append(s)
        o = oracle_lib.Session(omodel)
        o.feed(ids)
        oracles.append(o)
    batch = nb.Batch(model, sessions)
    for _ in range(3):
        got = batch.step()
        want = []
        for o in oracles:
            token = oracle_lib.argmax(o.logits())
            o.push(token)
            want.append(token)
        assert list(got) == want
    for s, o in zip(sessions, oracles):
        assert _bits_equal(s.logits(), o.logits())
    batch.close()
    for s in sessions:
        s.close()
    model.close()


def test_clone_shares_the_prefix_copy_on_write(device_model, oracle_model, oracle_lib):
    import rustyneedle_b200 as nb

    model = device_model.with_depth(2)
    base = nb.Session(model)
    base.feed(prompt_ids(7, 70))  # ends inside a partly filled page
    a, b = base.clone(), base.clone()
    a.push(11)
    b.push(12)
    o = oracle_lib.Session(oracle_model.with_depth(2))
    o.feed(prompt_ids(7, 70))
    oa, ob = o.clone(), o.clone()
    oa.push(11)
    ob.push(12)
    assert _bits_equal(a.logits(), oa.logits()) and _bits_equal(b.logits(), ob.logits())
    assert _bits_equal(base.logits(), o.logits())
    # the original steps after the clones, through batch steps: it was the
    # private owner of its last page before the clones shared it, so its next
    # write must copy that page first and leave the clones' positions alone
    batch = nb.Batch(model, [base])
    for _ in range(3):
        got = int(batch.step()[0])
        want = oracle_lib.argmax(o.logits())
        o.push(want)
        assert got == want
    batch.close()
    assert _bits_equal(base.logits(), o.logits())
    a.push(13)
    oa.push(13)
    b.push(14)
    ob.push(14)
    assert _bits_equal(a.logits(), oa.logits()) and _bits_equal(b.logits(), ob.logits())


def test_chunked_prefill_is_exact(archive_path, oracle_model, oracle_lib):
    import rustyneedle_b200 as nb

    model = nb.Model.open(archive_path, max_sessions=4, max_batch_tokens=96).with_depth(2)
    ids = prompt_ids(21, 300)
    s = nb.Session(model)
    s.feed(ids)
    stepped = nb.Session(model)
    for t in ids[:40]:
        stepped.push(int(t))
    stepped.feed(ids[40:])
    o = oracle_lib.Session(oracle_model.with_depth(2))
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits()) and _bits_equal(stepped.logits(), o.logits())


# ------------------------------------------------------------------ errors
def test_context_overflow_and_depth_errors(archive_path, device_model):
    import rustyneedle_b200 as nb

    with pytest.raises(nb.DepthError):
        device_model.with_depth(1)
    with pytest.raises(nb.DepthError):
        device_model.with_depth(21)
    model = device_model.with_depth(2)
    s = nb.Session(model)
    with pytest.raises(nb.ContextOverflow):
        s.feed(np.full(model.config.max_seq_len + 1, 10, dtype=np.uint32))
    assert len(s) == 0
    with pytest.raises(nb.NeedleError):
        s.push(model.config.vocab)


def test_kv_pool_exhaustion_is_a_status(archive_path):
    import rustyneedle_b200 as nb

    model = nb.Model.open(archive_path, max_sessions=2, kv_pages=4).with_depth(2)
    s = nb.Session(model)
    s.feed(prompt_ids(1, 64))  # one page per active layer
    with pytest.raises(nb.NeedleError) as err:
        s.feed(prompt_ids(2, 128))
    assert err.value.status == -8
