"""Device grammar masks (nb_token_automaton_*) against the CPU restatement of
TokenBytes::allowed / advance (crates/grammar/src/mask.rs:28-49) and run_turn's
constrained branch (crates/generate/src/generator.rs:102-124): mask words and
advanced states bit-exact on random automata (with rejected bytes that move
the state), and constrained greedy loops whose masks never leave the device
choosing the same ids as the same loops fed host masks from the restated
machines: a tool-name choice (the Name stage, call.rs:123-130) and whole tool
calls of the reference's home-assistant tools compiled by
nb_call_grammar_compile (CallMachine, call.rs:92-174)."""

import json
import os

import numpy as np
import pytest

from oracle import grammar as og
from tests.conftest import prompt_ids

pytestmark = pytest.mark.gpu

CALL_START, CALL_END = 1, 2
OPTIONS = [b"get_weather", b"get_time", b"search", b"send_mail", b"search_web"]


@pytest.fixture(scope="module")
def model(small_archive_path):
    import rustyneedle_b200 as nb

    m = nb.Model.open(small_archive_path)
    yield m
    m.close()


def _random_automaton(rng, states, vocab):
    alphabet = np.arange(97, 109)
    trans = np.zeros((states, 256), dtype=np.uint32)
    live = rng.random((states, alphabet.size)) < 0.7
    trans[:, alphabet] = np.where(live, rng.integers(1, states, size=(states, alphabet.size)), 0)
    # some rejected bytes change the state (the top bit), as array and object stages do
    moves = (trans == 0) & (rng.random((states, 256)) < 0.05)
    trans = np.where(moves, np.uint32(0x80000000) | rng.integers(1, states, size=(states, 256)).astype(np.uint32), trans)
    trans[0] = 0
    complete = (rng.random(states) < 0.05).astype(np.uint8)
    complete[0] = 0
    pieces = [None, None, None]
    for _ in range(vocab - 3):
        r = rng.random()
        if r < 0.85:
            pieces.append(bytes(rng.choice(alphabet, size=int(rng.integers(1, 7))).tolist()))
        elif r < 0.95:
            pieces.append(bytes(rng.integers(0, 256, size=int(rng.integers(1, 4))).tolist()))
        else:
            pieces.append(b"" if r < 0.975 else None)
    return trans, complete, pieces


def test_automaton_mask_and_advance_bit_exact(model):
    import torch

    import rustyneedle_b200 as nb

    V = model.config.output_vocab
    rng = np.random.default_rng(11)
    trans, complete, pieces = _random_automaton(rng, 61, V)
    start = 5 if not complete[5] else 6
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, CALL_START, CALL_END)
    B = 40
    states = rng.integers(0, 61, size=B).astype(np.uint32)
    states[:3] = 0
    states[3] = int(np.nonzero(complete)[0][0])
    d_states = torch.from_numpy(states.view(np.int32).copy()).cuda()
    d_mask = torch.full((B * V // 32,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()  # torch's fill runs on its own stream; the automaton on the model's
    aut.mask(d_states, d_mask)
    aut.check()
    got = d_mask.cpu().numpy().view(np.uint32).reshape(B, V // 32)
    for b in range(B):
        want = og.mask_words(og.automaton_mask(trans, complete, pieces, int(states[b]), CALL_END))
        assert np.array_equal(got[b], want), f"sequence {b} (state {states[b]})"
    nxt = rng.integers(0, V, size=B).astype(np.uint32)
    nxt[0], nxt[1], nxt[4], nxt[5], nxt[6] = CALL_START, 0xFFFFFFFF, CALL_END, CALL_START, 0xFFFFFFFF
    d_nxt = torch.from_numpy(nxt.view(np.int32).copy()).cuda()
    torch.cuda.synchronize()
    aut.advance(d_nxt, d_states)
    aut.check()
    after = d_states.cpu().numpy().view(np.uint32)
    for b in range(B):
        want = og.automaton_advance(trans, pieces, int(states[b]), int(nxt[b]), start, CALL_START, CALL_END)
        assert int(after[b]) == want, f"sequence {b}"
    aut.close()


def test_automaton_reports_out_of_range_state(model):
    import torch

    import rustyneedle_b200 as nb

    V = model.config.output_vocab
    trans, complete, start = nb.literal_automaton(OPTIONS)
    pieces = [None] * 3 + [bytes([97 + (t % 20)]) for t in range(3, V)]
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, CALL_START, CALL_END)
    d_states = torch.tensor([start, trans.shape[0] + 7], dtype=torch.int32, device="cuda")
    d_mask = torch.zeros(2 * V // 32, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    aut.mask(d_states, d_mask)
    with pytest.raises(nb.NeedleError):
        aut.check()
    aut.check()  # the report was cleared
    assert (d_mask.cpu().numpy().view(np.uint32)[V // 32:] == 0xFFFFFFFF).all()
    with pytest.raises(nb.NeedleError):
        nb.TokenAutomaton(model, trans, complete, start, pieces[:-32], CALL_START, CALL_END)
    bad = trans.copy()
    bad[1, 0] = trans.shape[0]
    with pytest.raises(nb.NeedleError):
        nb.TokenAutomaton(model, bad, complete, start, pieces, CALL_START, CALL_END)
    aut.close()


def test_constrained_loop_device_masks_match_host_masks(model):
    import torch

    import rustyneedle_b200 as nb

    V = model.config.output_vocab
    rng = np.random.default_rng(12)
    joined = b"|".join(OPTIONS)
    pieces = [None, None, None]
    while len(pieces) < V:
        if rng.random() < 0.7:
            a = int(rng.integers(0, len(joined)))
            pieces.append(joined[a:a + int(rng.integers(1, 4))])
        else:
            pieces.append(bytes(rng.integers(0, 256, size=int(rng.integers(1, 3))).tolist()))
    trans, complete, start = nb.literal_automaton(OPTIONS)
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, CALL_START, CALL_END)
    B = 4
    dev_sessions = []
    for b in range(B):
        s = nb.Session(model)
        s.feed(prompt_ids(300 + b, 40 + 9 * b))
        dev_sessions.append(s)
    host_sessions = [s.clone() for s in dev_sessions]
    dev_batch, host_batch = nb.Batch(model, dev_sessions), nb.Batch(model, host_sessions)
    first = [start, start, 0, start]
    d_states = torch.tensor(first, dtype=torch.int32, device="cuda")
    d_mask = torch.zeros(B * V // 32, dtype=torch.int32, device="cuda")
    d_next = torch.zeros(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    machines = [og.NameChoice(OPTIONS) if s else None for s in first]
    entered = 0
    for step in range(20):
        aut.mask(d_states, d_mask)
        dev_batch.step_device(d_mask.data_ptr(), d_next.data_ptr())
        aut.advance(d_next, d_states)
        aut.check()
        dev_ids = d_next.cpu().numpy().view(np.uint32)
        words = []
        for m in machines:
            if m is None:
                flags = [True] * V
            elif m.is_complete():
                flags = [t == CALL_END for t in range(V)]
            else:
                flags = og.allowed(pieces, m)
            words.append(og.mask_words(flags))
        host_ids = host_batch.step(np.concatenate(words))
        assert dev_ids.tolist() == host_ids.tolist(), f"step {step}"
        for b, t in enumerate(host_ids.tolist()):
            if t == CALL_START and machines[b] is None:
                machines[b] = og.NameChoice(OPTIONS)
            elif t == CALL_END:
                machines[b] = None
                entered += 1
            elif machines[b] is not None:
                og.advance(pieces, machines[b], t)
    assert entered > 0  # at least one call spelled out to the end under the device masks
    aut.close()


def test_tool_call_loop_device_masks_match_host_masks(model):
    """Whole tool calls: the reference's home-assistant tools (object arguments,
    enums, bounded integers, a choice) compiled by nb_call_grammar_compile; four
    sequences start inside a call (tool_call_start pushed) and step 40 times
    with masks and advances on the device only, beside the same batch stepped
    with host masks from the restated CallMachine and TokenBytes::allowed."""
    import torch

    import rustyneedle_b200 as nb

    V = model.config.output_vocab
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tool_schemas.json")
    with open(path) as f:
        tools = json.load(f)["home_assistant.json"]
    rng = np.random.default_rng(21)
    text = json.dumps(tools).encode() + b'[{"name":"' + b',"arguments":{' + b'0123456789}],'
    pieces = [None, None, None] + [bytes([b]) for b in range(256)]
    while len(pieces) < V:
        a = int(rng.integers(0, len(text)))
        pieces.append(text[a:a + int(rng.integers(1, 8))])
    trans, complete, start = nb.call_automaton(tools)
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, CALL_START, CALL_END)
    grammar = og.CallGrammar(tools)
    B = 4
    dev_sessions = []
    for b in range(B):
        s = nb.Session(model)
        s.feed(prompt_ids(700 + b, 24 + 7 * b))
        dev_sessions.append(s)
    host_sessions = [s.clone() for s in dev_sessions]
    dev_batch, host_batch = nb.Batch(model, dev_sessions), nb.Batch(model, host_sessions)
    d_states = torch.full((B,), start, dtype=torch.int32, device="cuda")
    d_mask = torch.zeros(B * V // 32, dtype=torch.int32, device="cuda")
    d_next = torch.zeros(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    machines = [grammar.start() for _ in range(B)]
    deepest = 0
    for step in range(40):
        aut.mask(d_states, d_mask)
        dev_batch.step_device(d_mask.data_ptr(), d_next.data_ptr())
        aut.advance(d_next, d_states)
        aut.check()
        dev_ids = d_next.cpu().numpy().view(np.uint32)
        words = []
        for m in machines:
            if m is None:
                flags = [True] * V
            elif m.is_complete():
                flags = [t == CALL_END for t in range(V)]
            else:
                flags = og.allowed(pieces, m)
            words.append(og.mask_words(flags))
        host_ids = host_batch.step(np.concatenate(words))
        assert dev_ids.tolist() == host_ids.tolist(), f"step {step}"
        for b, t in enumerate(host_ids.tolist()):
            if t == CALL_START and machines[b] is None:
                machines[b] = grammar.start()
            elif t == CALL_END:
                machines[b] = None
            elif machines[b] is not None:
                og.advance(pieces, machines[b], t)
                stages = ["open", "after_open", "prefix", "name", "middle", "arguments", "close", "after_call", "done"]
                deepest = max(deepest, stages.index(machines[b].stage[0]))
    assert deepest >= 5  # some sequence chose a tool and entered its arguments under the device masks
    aut.close()
