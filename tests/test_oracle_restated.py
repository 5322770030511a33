"""The C++ restatement (oracle/needle_oracle.cpp, INT mode) against a second,
independent numpy restatement written from the reference's Rust
(oracle/restated.py), on the composite paths that no reference test vector
pins: codebook products with their per-group combine, one head's attention
with 12-bit value weights, the Sinkhorn mixing, the grammar step's allowed
statistics, and, with the archive's own weights, a layer's Hadamard block,
its lane routing, whole tokens (every layer's lane stream, then the logits)
and Whistle tokens with their cross memory. Seeded random inputs;
bit-exact. CPU only."""

from fractions import Fraction

import numpy as np
import pytest

from oracle import restated


def _exact_f32(value: Fraction) -> np.float32:
    """Round an exact rational to the nearest f32 (ties to even)."""
    if value == 0:
        return np.float32(0.0)
    sign = -1 if value < 0 else 1
    a = abs(value)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    k = max(e - 23, -149)  # the f32 spacing at this magnitude
    q = a / Fraction(2) ** k
    n = q.numerator // q.denominator
    r = q - n
    if r > Fraction(1, 2) or (r == Fraction(1, 2) and n % 2 == 1):
        n += 1
    return np.float32(sign * float(n * Fraction(2) ** k))


def test_fused_multiply_add_rounds_once():
    rng = np.random.default_rng(5)
    a = rng.standard_normal(3000).astype(np.float32) * np.float32(1000)
    b = rng.standard_normal(3000).astype(np.float32) * np.float32(1e-3)
    c = rng.standard_normal(3000).astype(np.float32)
    # halfway cases: c + (an exact f32 half-ulp) + a tiny product of the other sign
    ulp = np.spacing(np.float32(1.0))
    a[:4] = [np.float32(ulp / 2), np.float32(ulp / 2), np.float32(ulp / 2), np.float32(ulp / 2)]
    b[:4] = [np.float32(1.0) + np.float32(2.0**-20), np.float32(1.0) - np.float32(2.0**-21), 1.0, -1.0]
    c[:4] = [1.0, 1.0, 1.0, 1.0]
    got = restated.fma_f32(a, b, c)
    for i in range(a.size):
        want = _exact_f32(Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i])))
        assert got[i] == want, (i, a[i], b[i], c[i], got[i], want)


def _levels(rng, bits):
    half = np.sort(np.abs(rng.standard_normal(1 << (bits - 1)))).astype(np.float32) + np.float32(0.05)
    return np.concatenate([-half[::-1], half]).astype(np.float32)


@pytest.mark.parametrize("bits,rows,cols", [(2, 96, 512), (2, 37, 1024), (4, 64, 512), (4, 33, 2048)])
def test_codebook_products(oracle_lib, bits, rows, cols):
    rng = np.random.default_rng(bits * 1000 + rows)
    packed = rng.integers(0, 256, rows * cols * bits // 8, dtype=np.uint8)
    levels = _levels(rng, bits)
    norms = (rng.uniform(1e-3, 2e-2, rows * (cols // 128))).astype(np.float16).view(np.uint16)
    for trial in range(3):
        x = rng.standard_normal(cols).astype(np.float32) * np.float32(3.0 ** trial)
        if trial == 2:
            x[128:256] = 0.0  # a zero group: activation scale 1
        want = oracle_lib.product_raw(oracle_lib.MODE_INT, bits, packed, levels, norms, rows, cols, x)
        got = restated.product_int(bits, packed, levels, norms, rows, cols, x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (bits, trial, np.flatnonzero(got != want)[:5])


@pytest.mark.parametrize("count", [1, 3, 4, 5, 63, 64, 257, 1000, 2048])
def test_attention_head(oracle_lib, count):
    rng = np.random.default_rng(count)
    dim = 64
    for trial in range(3):
        q = rng.integers(-127, 128, dim).astype(np.int8)
        keys = rng.integers(-127, 128, (count, dim)).astype(np.int8)
        values = rng.integers(-127, 128, (count, dim)).astype(np.int8)
        ks = rng.uniform(1e-3, 3e-2, count).astype(np.float32)
        vs = rng.uniform(1e-3, 3e-2, count).astype(np.float32)
        qs = np.float32(rng.uniform(1e-3, 2e-2) / 8.0)
        if trial == 2:
            ks[: count // 2] *= np.float32(10.0)  # a sharper softmax: many weights round to zero
        want = oracle_lib.attend_head_raw(oracle_lib.MODE_INT, q, qs, keys, ks, values, vs)
        got = restated.attend_head_int(q, qs, keys, ks, values, vs)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (count, trial, np.flatnonzero(got != want)[:5])


def test_sinkhorn(oracle_lib):
    rng = np.random.default_rng(9)
    for trial in range(20):
        logits = (rng.standard_normal(16) * (0.5 + trial)).astype(np.float32)
        want = oracle_lib.sinkhorn(logits, 4)
        got = restated.sinkhorn(logits, 4)
        assert np.array_equal(np.asarray(got).view(np.uint32), np.asarray(want, dtype=np.float32).view(np.uint32)), trial


def test_allowed_statistics(oracle_lib):
    rng = np.random.default_rng(13)
    vocab = 8192
    for trial in range(6):
        logits = (rng.standard_normal(vocab) * (1.0 + 3 * trial)).astype(np.float32)
        allowed = rng.random(vocab) < (0.05 if trial % 2 else 0.6)
        allowed[rng.integers(0, vocab)] = True
        ids = np.flatnonzero(allowed)
        token = int(ids[rng.integers(0, ids.size)])
        want = oracle_lib.allowed_statistics(logits, token, allowed)
        got = restated.allowed_statistics(logits, token, allowed)
        assert np.float32(want[0]) == got[0] and np.float32(want[1]) == got[1], (trial, want, got)


def test_archive_reader_sees_the_layout(small_archive_path):
    arch = restated.Archive(small_archive_path)
    t = arch.hadamard(3)
    n = t["d1"].size
    assert n == 2048 and t["w1a"].size == 64 * 64 and t["w1b"].size == 32 * 32 and t["cond_v"].size == 512 * 8
    assert t["cond_u"].size == 8 * n and sorted(t["perms"][0]) == list(range(n))
    lt = arch.lane_tensors()
    assert lt["a_pre"].size == arch.layers and lt["phi_res"][4] == arch.layers * arch.lanes * arch.lanes


@pytest.mark.parametrize("layer", [0, 3])
def test_hadamard_block(oracle_lib, small_archive_path, layer):
    """HadamardWeights::apply with the archive's factors, read by each
    restatement's own archive reader."""
    arch = restated.Archive(small_archive_path)
    model = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT)
    rng = np.random.default_rng(40 + layer)
    t = arch.hadamard(layer)
    for trial in range(3):
        x = (rng.standard_normal(arch.d_model) * (0.3 + trial)).astype(np.float32)
        want = model.hadamard(layer, x)
        got = restated.hadamard_apply(t, x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (layer, trial, np.flatnonzero(got != want)[:5])


@pytest.mark.parametrize("layer,slot", [(0, 0), (1, 5), (3, 2)])
def test_routing(oracle_lib, small_archive_path, layer, slot):
    """LaneWeights::route: the phi products through the archive's 4-bit lane
    maps, the gates with the session's own-lane offsets, the Sinkhorn."""
    arch = restated.Archive(small_archive_path)
    model = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT)
    lt = arch.lane_tensors()
    rng = np.random.default_rng(70 + layer * 8 + slot)
    for trial in range(3):
        stream = (rng.standard_normal(arch.lanes * arch.d_model) * (0.5 + trial)).astype(np.float32)
        want = model.route(layer, slot, stream)
        got = restated.route(lt, arch.lanes, layer, slot, stream)
        for name, g, w in zip(("input", "post", "residual"), got, want):
            assert np.array_equal(np.asarray(g, dtype=np.float32).view(np.uint32), w.view(np.uint32)), (name, trial)


def test_whole_tokens(oracle_lib, small_archive_path):
    """Session::push and Session::logits end to end (4 layers): the lane
    stream after every layer for six tokens, then the logits."""
    arch = restated.Archive(small_archive_path)
    model = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT)
    ours, theirs = restated.Session(arch), oracle_lib.Session(model)
    for position, token in enumerate([17, 300, 5000, 42, 9, 1234]):
        want = theirs.push_traced(token)
        got = ours.push(token)
        for layer in range(arch.layers):
            w, g = want[layer].reshape(-1), got[layer]
            assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), (position, layer, np.flatnonzero(g != w)[:5])
    want, got = theirs.logits(), ours.logits()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.flatnonzero(got != want)[:5]


def test_whistle_cross_attention(oracle_lib):
    """CrossWeights::memory and CrossState::apply inside Session::push_with on
    a 4-layer synthetic Whistle archive: the logits after bos, a language
    token and three text tokens, with a 48-frame encoder output."""
    from rustyneedle_b200 import synthetic

    path = synthetic.cached_archive(seed=19, geometry=synthetic.Geometry(num_layers=4, max_seq_len=512, text_vocab=8000))
    arch = restated.Archive(path)
    model = oracle_lib.Model.open(path, oracle_lib.MODE_INT)
    encoded = np.random.default_rng(23).standard_normal((48, arch.d_model)).astype(np.float32)
    ours = restated.Session(arch)
    memory = restated.cross_memory(arch, encoded, ours.heads, ours.head_dim)
    theirs = oracle_lib.Session(model)
    theirs_memory = oracle_lib.CrossMemory(model, encoded)
    for layer in (0, 3):  # the memory itself (keys, values and their scales)
        k, ks, v, vs = theirs_memory.read(layer, ours.heads)
        assert np.array_equal(np.asarray(k).reshape(memory[layer]["keys"].shape), memory[layer]["keys"])
        assert np.array_equal(np.asarray(v).reshape(memory[layer]["values"].shape), memory[layer]["values"])
        assert np.array_equal(np.asarray(ks, dtype=np.float32).reshape(-1).view(np.uint32), memory[layer]["key_scales"].reshape(-1).view(np.uint32))
        assert np.array_equal(np.asarray(vs, dtype=np.float32).reshape(-1).view(np.uint32), memory[layer]["value_scales"].reshape(-1).view(np.uint32))
    for token in [1, 8003, 17, 4242, 99]:
        theirs.push_cross(token, theirs_memory)
        ours.push(token, memory)
        want, got = theirs.logits(), ours.logits()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (token, np.flatnonzero(got != want)[:5])


def test_prefill_against_pushes(oracle_lib, small_archive_path):
    """Session::feed of 20 tokens (the prefill path, prefill.rs:10-99, in the
    C++ restatement) against the numpy restatement pushing them one by one:
    the logits and every layer's int8 cache."""
    arch = restated.Archive(small_archive_path)
    model = oracle_lib.Model.open(small_archive_path, oracle_lib.MODE_INT)
    tokens = [int(t) for t in np.random.default_rng(3).integers(10, 8000, 20)]
    theirs = oracle_lib.Session(model)
    theirs.feed(tokens)
    ours = restated.Session(arch)
    for token in tokens:
        ours.push(token)
    assert np.array_equal(ours.logits().view(np.uint32), theirs.logits().view(np.uint32))
    for layer in range(arch.layers):
        keys, key_scales, values, value_scales = theirs.cache(layer)
        cache = ours.caches[layer]
        assert np.array_equal(np.stack(cache["keys"]), keys) and np.array_equal(np.stack(cache["values"]), values)
        assert np.array_equal(np.array(cache["key_scales"], dtype=np.float32).view(np.uint32), key_scales.view(np.uint32))
        assert np.array_equal(np.array(cache["value_scales"], dtype=np.float32).view(np.uint32), value_scales.view(np.uint32))


def test_conv_taps_and_sliding_window(oracle_lib):
    """Whole tokens on an archive with 3-tap q/k/v convolutions and a 40-position
    sliding window on every layer but the first and last (global): 50 tokens,
    so the window and the taps' history both fill; every layer's lane stream
    at every tenth token, then the logits."""
    from rustyneedle_b200 import synthetic

    geometry = synthetic.Geometry(num_layers=6, max_seq_len=512, conv_taps=3, sliding_window=40, global_layers=0b100001)
    path = synthetic.cached_archive(seed=7, geometry=geometry)
    arch = restated.Archive(path)
    model = oracle_lib.Model.open(path, oracle_lib.MODE_INT)
    ours, theirs = restated.Session(arch), oracle_lib.Session(model)
    for position, token in enumerate(np.random.default_rng(5).integers(10, 8000, 50)):
        want = theirs.push_traced(int(token))
        got = ours.push(int(token))
        if position % 10 == 9:
            for layer in range(arch.layers):
                w, g = want[layer].reshape(-1), got[layer]
                assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), (position, layer, np.flatnonzero(g != w)[:5])
    want, got = theirs.logits(), ours.logits()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.flatnonzero(got != want)[:5]


def test_engram_sites(oracle_lib):
    """Whole tokens on an archive with engram sites at layers 1 and 4 (orders
    2 and 3, two hashed tables per order, a 3-tap dilation-2 value
    convolution) besides conv taps and sliding windows: 30 tokens, every
    layer's lane stream at every fifth token, then the logits."""
    from rustyneedle_b200 import synthetic

    geometry = synthetic.Geometry(num_layers=6, max_seq_len=512, conv_taps=3, sliding_window=40, global_layers=0b100001,
                                  engram_sites=(1, 4), engram_slots=512, engram_orders=(2, 3), engram_heads_per_order=2,
                                  engram_conv_taps=3, engram_dilation=2)
    path = synthetic.cached_archive(seed=11, geometry=geometry)
    arch = restated.Archive(path)
    assert arch.engram["sites"] == [1, 4] and arch.engram["orders"] == [2, 3]
    model = oracle_lib.Model.open(path, oracle_lib.MODE_INT)
    ours, theirs = restated.Session(arch), oracle_lib.Session(model)
    for position, token in enumerate(np.random.default_rng(6).integers(10, 8000, 30)):
        want = theirs.push_traced(int(token))
        got = ours.push(int(token))
        if position % 5 == 4 or position < 3:
            for layer in range(arch.layers):
                w, g = want[layer].reshape(-1), got[layer]
                assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), (position, layer, np.flatnonzero(g != w)[:5])
    want, got = theirs.logits(), ours.logits()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.flatnonzero(got != want)[:5]


def test_probe_heads(oracle_lib):
    """Probe heads (codes 2 and 3, two probes per cell, two queries, three
    outputs) on the engram/taps/window archive: the pooled readout and the
    head output after each of 12 tokens."""
    from rustyneedle_b200 import synthetic

    geometry = synthetic.Geometry(num_layers=6, max_seq_len=512, conv_taps=3, sliding_window=40, global_layers=0b100001,
                                  engram_sites=(1, 4), engram_slots=512, engram_orders=(2, 3), engram_heads_per_order=2,
                                  engram_conv_taps=3, engram_dilation=2, probe_heads=(2, 3), probes_per_layer=2, head_queries=2,
                                  head_outputs=3)
    path = synthetic.cached_archive(seed=16, geometry=geometry)
    arch = restated.Archive(path)
    model = oracle_lib.Model.open(path, oracle_lib.MODE_INT)
    ours, theirs = restated.Session(arch), oracle_lib.Session(model)
    assert [h.code for h in ours.heads_list] == [2, 3]
    for position, token in enumerate(np.random.default_rng(8).integers(10, 8000, 12)):
        theirs.push(int(token))
        ours.push(int(token))
        for code in (2, 3):
            for name in ("pooled_readout", "head_output"):
                want = np.asarray(getattr(theirs, name)(code), dtype=np.float32)
                got = getattr(ours, name)(code)
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (position, code, name, np.flatnonzero(got != want)[:5])
    assert ours.head_output(1) is None and theirs.head_output(1) is None
    want, got = theirs.logits(), ours.logits()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
