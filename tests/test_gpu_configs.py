"""Parity at the benchmark configurations' own sizes, through the C ABI,
against the CPU restatement in INT mode (the reference's integer kernels).

Each test decodes exactly the workload `bench.py` times (the generators in
rustyneedle_b200.workloads) and requires identical greedy tokens at every
step and bit-identical logits at the end (generator.rs:99-130 over
session.rs:56-148):

  config 1  depth 20, a 512-token prompt, 256 steps under the per-step 5 % bitsets
  config 2  four of rank 0's own sequences (the longest and the shortest among
            them) decoded for 32 steps inside the 256-sequence batch, so the
            two-chain step graph of batches of at least 256 runs
  config 4  two of the 64 utterances (depth 8, 1500-frame cross memories)
            over all 224 greedy text tokens, decoded inside the 64-batch
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    a, b = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _first_difference(got, want):
    got, want = np.asarray(got), np.asarray(want)
    bad = np.argwhere(got != want)
    return "equal" if bad.size == 0 else f"first difference at {tuple(bad[0])}: {got[tuple(bad[0])]} vs {want[tuple(bad[0])]}"


def test_config1_at_full_size(native_built, archive_path, oracle_lib):
    """Config 1 exactly: depth 20, 512-token prompt in one prefill, then 256
    greedy steps through nb_batch_step, each under its seeded ~5 % bitset,
    with allowed_statistics (generator.rs:182-194) held to 1e-6 relative."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import workloads

    model = nb.Model.open(archive_path, max_sessions=2)
    assert model.config.num_layers == workloads.CONFIG1["depth"]
    V = model.config.output_vocab
    ids, words, allowed = workloads.config1(V)
    s = nb.Session(model)
    s.feed(ids)
    omodel = oracle_lib.Model.open(archive_path, oracle_lib.MODE_INT, 0)
    o = oracle_lib.Session(omodel)
    o.feed(ids)
    assert _bits_equal(s.logits(), o.logits())
    batch = nb.Batch(model, [s])
    got, want = [], []
    for k in range(len(words)):
        token, stats = batch.step(words[k], stats=True)
        logits = o.logits()
        w = oracle_lib.argmax_allowed(logits, allowed[k].astype(np.uint8))
        p, m = oracle_lib.allowed_statistics(logits, w, allowed[k].astype(np.uint8))
        assert abs(stats[0].probability - p) <= 1e-6 * abs(p) and abs(stats[0].mass - m) <= 1e-6 * abs(m), k
        o.push(w)
        got.append(int(token[0]))
        want.append(w)
        assert got[-1] == w, f"step {k}: device {got[-1]}, oracle {w}"
    assert len(got) == 256 and len(s) == len(o) == 512 + 256
    assert _bits_equal(s.logits(), o.logits())
    batch.close()
    s.close()
    model.close()


def test_config2_sequences_inside_the_256_batch(native_built, archive_path, oracle_lib):
    """Config 2: rank 0's 256 sequences (prompts uniform in [128, 1024]) fed in
    shared prefill passes and stepped as one batch (two step groups of 128);
    four of them, the longest and the shortest included, against the oracle
    over 32 greedy steps."""
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import dp, workloads

    steps = 32
    prompts = workloads.config2_prompts(0)
    assert len(prompts) == 256
    pages = dp.kv_pages_for(prompts, steps + 4, 20)
    model = nb.Model.open(archive_path, max_sessions=len(prompts), kv_pages=pages)
    sessions = [nb.Session(model) for _ in prompts]
    nb.feed_many(sessions, prompts)
    batch = nb.Batch(model, sessions)
    tokens = np.stack([batch.step() for _ in range(steps)])  # [steps][256]

    lengths = np.array([len(p) for p in prompts])
    picked = [int(np.argmax(lengths)), int(np.argmin(lengths)), 77, 200]
    assert lengths[picked[0]] > 1000
    omodel = oracle_lib.Model.open(archive_path, oracle_lib.MODE_INT, 0)
    oracles = []
    for i in picked:
        o = oracle_lib.Session(omodel)
        o.feed(prompts[i])
        oracles.append(o)
    want = np.zeros((steps, len(picked)), dtype=np.uint32)
    want[0] = [oracle_lib.argmax(o.logits()) for o in oracles]
    for k in range(1, steps):
        logits = oracle_lib.sessions_step(oracles, want[k - 1])
        want[k] = [oracle_lib.argmax(row) for row in logits]
    final = oracle_lib.sessions_step(oracles, want[steps - 1])
    got = tokens[:, picked]
    assert np.array_equal(got, want), _first_difference(got, want)
    for j, i in enumerate(picked):
        assert len(sessions[i]) == len(prompts[i]) + steps
        assert _bits_equal(sessions[i].logits(), final[j]), i
    batch.close()
    for s in sessions:
        s.close()
    model.close()


def test_config4_utterances_inside_the_64_batch(native_built, oracle_lib):
    """Config 4: the depth-8 Whistle decoder, 64 utterances each with its own
    1500-frame cross memory, bos and a language token, then all 224 greedy
    text tokens (device-resident steps under the text-vocabulary mask); the
    first and the last utterance against the oracle."""
    import torch

    import rustyneedle_b200 as nb
    from rustyneedle_b200 import workloads

    W = workloads.WHISTLE
    archive = workloads.whistle_archive()
    model = nb.Model.open(archive, max_sessions=W["batch"])
    V = model.config.output_vocab
    encoded = list(workloads.whistle_encoded(W["batch"], model.config.d_model))
    sessions, memories = [], []
    for i, enc in enumerate(encoded):
        mem = nb.CrossMemory(model, enc)
        s = nb.Session(model)
        s.set_cross(mem)
        s.push(W["bos"])
        s.push(workloads.whistle_language(i, V))
        sessions.append(s)
        memories.append(mem)
    T, B = W["tokens"], W["batch"]
    masks = torch.from_numpy(np.tile(workloads.text_words(V), T * B).view(np.int32)).cuda()
    out = torch.zeros(T * B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    batch = nb.Batch(model, sessions)
    batch.run(T, masks.data_ptr(), out.data_ptr())
    tokens = out.cpu().numpy().view(np.uint32).reshape(T, B)

    omodel = oracle_lib.Model.open(archive, oracle_lib.MODE_INT, 0)
    allowed = workloads.text_allowed(V).astype(np.uint8)
    for i in (0, B - 1):
        omem = oracle_lib.CrossMemory(omodel, encoded[i])
        o = oracle_lib.Session(omodel)
        o.push_cross(W["bos"], omem)
        o.push_cross(workloads.whistle_language(i, V), omem)
        want = []
        for _ in range(T):
            t = oracle_lib.argmax_allowed(o.logits(), allowed)
            o.push_cross(t, omem)
            want.append(t)
        assert np.array_equal(tokens[:, i], want), (i, _first_difference(tokens[:, i], np.array(want)))
        assert _bits_equal(sessions[i].logits(), o.logits()), i
    batch.close()
    for s in sessions:
        s.close()
    for m in memories:
        m.close()
    model.close()
