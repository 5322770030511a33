"""The tool-call grammar compiled by the library (nb_call_grammar_compile)
against the CPU restatement of the reference's grammar crate
(oracle/grammar.py: CallGrammar, CallMachine and every machine form of
crates/grammar/src/{call,machine,schema}.rs). CPU only.

Along seeded random walks through each grammar — mostly accepted bytes, now
and then a rejected one, which some stages answer by changing state — every
automaton state must accept exactly the bytes the restated machine accepts,
move where it moves (also on a rejected byte that changes it), be complete
exactly when CallMachine::is_complete, and give TokenBytes::allowed's mask
over a vocabulary of multi-byte pieces. The grammars are the reference's own
example tool files (tests/golden/tool_schemas.json, extracted by
make_tool_schemas.py) and schemas written here for the forms those files do
not use (arrays, bounded numbers and texts, nested objects, $ref, const,
type lists, escapes, non-ASCII)."""

import json
import os
import zlib

import numpy as np
import pytest

from oracle import grammar as og
from rustyneedle_b200.grammar import call_automaton, literal_automaton

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tool_schemas.json")
CALL_START, CALL_END = 1, 2
TOP = 0x80000000

EXTRA = {
    "arrays_and_numbers": [
        {"name": "plot", "parameters": {"type": "object", "properties": {
            "points": {"type": "array", "items": {"type": "object", "properties": {
                "x": {"type": "number", "minimum": -2.5, "maximum": 100.75},
                "y": {"type": "integer", "exclusiveMinimum": -3, "maximum": 12}}, "required": ["x"]},
                "minItems": 1, "maxItems": 3},
            "scale": {"type": "number"},
            "label": {"type": "string", "minLength": 2, "maxLength": 5}}, "required": ["points", "label"]}},
        {"name": "plot_all", "parameters": {"type": "object", "properties": {
            "tags": {"type": "array", "items": {"type": "string", "enum": ["a", "ab", "b\"q"]}, "maxItems": 2},
            "on": {"type": "boolean"}, "none": {"type": "null"}}}},
    ],
    "refs_consts_choices": [
        {"function": {"name": "book", "parameters": {
            "type": "object", "$defs": {"when": {"type": "string", "maxLength": 4}},
            "properties": {
                "when": {"$ref": "#/$defs/when"},
                "kind": {"const": "table"},
                "seats": {"type": ["integer", "null"], "minimum": 1, "maximum": 8},
                "note": {"anyOf": [{"type": "string", "maxLength": 2}, {"type": "number", "minimum": 0, "maximum": 1}]},
                "city": {"enum": ["Zürich", "Köln", 3, 2.5, True, None]}},
            "required": ["when", "kind"]}}},
        {"name": "noop"},
        {"name": "free", "parameters": {"type": "string"}},
    ],
}


def _grammars():
    with open(GOLDEN) as f:
        fixtures = json.load(f)
    cases = [(name, tools) for name, tools in sorted(fixtures.items())]
    return cases + sorted(EXTRA.items())


def _structural(rng):
    return int(rng.choice(list(b'"}]:,{[0123456789.-tfnul \\')))


def _walk(trans, complete, start, grammar, rng, steps=260, rejected=0.08, check_rejected=6):
    """One random walk; asserts the automaton follows the restated machine."""
    m, s = grammar.start(), start
    for _ in range(steps):
        assert bool(complete[s]) == m.is_complete()
        row = trans[s]
        accepted = []
        moved = []
        for b in range(256):
            c = m.clone()
            ok = c.step(b)
            t = int(row[b])
            assert ok == (t != 0 and not t & TOP), (b, t)
            if ok:
                accepted.append((b, c))
            elif t & TOP:
                moved.append((b, c, t & ~TOP))
        # a rejected byte that changes the machine: the automaton's target behaves as the changed machine
        for b, c, target in moved[:check_rejected]:
            for b2 in rng.choice(256, 24, replace=False):
                t2 = int(trans[target, b2])
                assert c.clone().step(int(b2)) == (t2 != 0 and not t2 & TOP), (b, b2)
        if m.is_complete() or not accepted:
            return
        if rng.random() < rejected:
            b = int(rng.integers(0, 256))
            t = int(row[b])
            if t == 0 or t & TOP:
                m.step(b)
                s = t & ~TOP if t & TOP else s
                continue
        if rng.random() < 0.45:
            pick = _structural(rng)
            hit = [x for x in accepted if x[0] == pick]
            b, c = hit[0] if hit else accepted[int(rng.integers(0, len(accepted)))]
        else:
            b, c = accepted[int(rng.integers(0, len(accepted)))]
        m, s = c, int(row[b])


@pytest.mark.parametrize("name,tools", _grammars(), ids=[n for n, _ in _grammars()])
def test_compiled_call_grammar_follows_the_call_machine(name, tools):
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    variants = [(False, None), (True, None), (True, [len(tools) - 1, 0] if len(tools) > 1 else [0])]
    for require, permitted in variants:
        trans, complete, start = call_automaton(tools, require, permitted)
        assert trans.shape[0] == complete.shape[0] and trans.shape[0] < 20000
        assert complete[0] == 0 and not trans[0].any()
        grammar = og.CallGrammar(tools, require, permitted)
        for _ in range(3):
            _walk(trans, complete, start, grammar, rng)


def _pieces(tools, rng, count=420):
    """Vocabulary pieces: the single bytes of the call syntax, substrings of the
    tools JSON (names, keys, enum values), random bytes, None and empty."""
    text = json.dumps(tools).encode() + b'[{"name":"' + b',"arguments":' + b'0123456789.-'
    pieces = [None, None, None] + [bytes([b]) for b in b'[]{}":,0123456789.- abcdefghijklmnopqrstuvwxyz']
    while len(pieces) < count:
        r = rng.random()
        if r < 0.75:
            a = int(rng.integers(0, len(text)))
            pieces.append(text[a:a + int(rng.integers(1, 7))])
        elif r < 0.95:
            pieces.append(bytes(rng.integers(0, 256, size=int(rng.integers(1, 4))).tolist()))
        else:
            pieces.append(b"" if r < 0.975 else None)
    return pieces


@pytest.mark.parametrize("name,tools", _grammars()[:3] + _grammars()[-2:], ids=[n for n, _ in _grammars()[:3] + _grammars()[-2:]])
def test_masks_and_advance_over_pieces(name, tools):
    """TokenBytes::allowed / advance (mask.rs:28-49) along greedy-like walks
    that pick allowed pieces: the automaton's masks and advanced states equal
    the restated machine's; after a complete call only call_end is allowed."""
    rng = np.random.default_rng(7 + len(name))
    pieces = _pieces(tools, rng)
    trans, complete, start = call_automaton(tools)
    grammar = og.CallGrammar(tools)
    for _ in range(3):
        m, s = grammar.start(), start
        for _ in range(40):
            want = [t == CALL_END for t in range(len(pieces))] if m.is_complete() else og.allowed(pieces, m)
            got = og.automaton_mask(trans, complete, pieces, s, CALL_END)
            assert got == want
            if m.is_complete():
                assert og.automaton_advance(trans, pieces, s, CALL_END, start, CALL_START, CALL_END) == 0
                break
            ids = [t for t, ok in enumerate(want) if ok]
            if not ids:
                break
            # mostly allowed pieces, sometimes any piece (the unrestricted fallback, generator.rs:107)
            token = int(rng.choice(ids)) if rng.random() < 0.9 else int(rng.integers(3, len(pieces)))
            og.advance(pieces, m, token)
            s = og.automaton_advance(trans, pieces, s, token, start, CALL_START, CALL_END)
            assert bool(complete[s]) == m.is_complete()


def test_a_whole_call_reaches_completion():
    tools = EXTRA["refs_consts_choices"]
    trans, complete, start = call_automaton(tools)
    text = b'[{"name":"book","arguments":{"when":"mon","kind":"table","seats":null,"city":"K\xc3\xb6ln"}},' \
           b'{"name":"noop","arguments":{}}]'
    m, s = og.CallGrammar(tools).start(), start
    for b in text:
        assert m.step(b)
        t = int(trans[s, b])
        assert t and not t & TOP
        s = t
    assert m.is_complete() and complete[s]
    # an empty call list is allowed unless a call is required (call.rs:99-102)
    assert trans[int(trans[start, ord("[")]), ord("]")] != 0
    t2, c2, s2 = call_automaton(tools, require_call=True, permitted=[2])
    assert t2[int(t2[s2, ord("[")]), ord("]")] == 0


def test_literal_automaton_follows_the_name_stage():
    """A name that is a prefix of another is chosen as soon as it has ended
    (call.rs:123-130): its node is complete and nothing beneath it is reachable."""
    options = [b"get", b"get_user", b"search", b"s"]
    for permitted in (None, [1, 2], [2, 0]):
        trans, complete, start = literal_automaton(options, permitted)
        rng = np.random.default_rng(1)
        for _ in range(40):
            m, s = og.NameChoice(options, permitted), start
            for _ in range(10):
                assert bool(complete[s]) == m.is_complete()
                for b in range(256):
                    assert m.clone().step(b) == (trans[s, b] != 0)
                ok = [b for b in range(256) if trans[s, b]]
                if not ok:
                    break
                b = int(rng.choice(ok))
                m.step(b)
                s = int(trans[s, b])
    trans, complete, start = literal_automaton(options)
    s = start
    for b in b"get":
        s = int(trans[s, b])
    assert complete[s] and not trans[s].any()  # "get" chosen; "get_user" unreachable
    s = int(trans[start, ord("s")])
    assert complete[s]  # "s" chosen before "search" could continue


def test_compile_errors_are_statuses():
    import rustyneedle_b200 as nb

    with pytest.raises(nb.NeedleError) as e:
        call_automaton('[{"name": "x", ')
    assert e.value.status == -4
    with pytest.raises(nb.NeedleError) as e:
        call_automaton([{"name": "x"}], require_call=True, permitted=[3])
    assert e.value.status == -4
    with pytest.raises(nb.NeedleError) as e:
        call_automaton([{"name": "x"}], require_call=False, permitted=[0])
    assert e.value.status == -4
    with pytest.raises(nb.NeedleError) as e:
        call_automaton(EXTRA["arrays_and_numbers"], max_states=50)
    assert e.value.status == -5
    # tools without a string name are skipped (call.rs:22-24); no tools: only "[]"
    trans, complete, start = call_automaton([{"parameters": {}}, {"name": 3}])
    after = int(trans[start, ord("[")])
    assert complete[int(trans[after, ord("]")])]


def test_literal_text_matches_serde_json():
    """serde_json::to_string of const/enum values (schema.rs:51-53)."""
    assert og.literal_text(["a\"b\\", "é\n\x01", 1, -7, 2.5, 1e20, 1e-7, 0.1, 100.0, 1e16, 123456.789, True, None]) == \
        '["a\\"b\\\\","é\\n\\u0001",1,-7,2.5,1e20,1e-7,0.1,100.0,1e16,123456.789,true,null]'
