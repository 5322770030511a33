"""Device grammar masks, host side: the trie automaton that literal_automaton
compiles reproduces a call's tool-name choice (the Name stage of
CallMachine::step over LiteralState, crates/grammar/src/call.rs:123-130,
machine.rs:278-312) under TokenBytes::allowed / advance
(crates/grammar/src/mask.rs:28-49) along random constrained walks, and the
automaton's marker rules follow run_turn (crates/generate/src/generator.rs:102-124).
CPU only."""

import numpy as np

from oracle import grammar as og
from rustyneedle_b200.grammar import literal_automaton, token_table

OPTIONS = [b"get_weather", b"get_time", b"search", b"send_mail", b"s", b"search_web"]
CALL_START, CALL_END = 1, 2


def _pieces(rng, count):
    """Vocabulary pieces: substrings of the options, random bytes, None and empty."""
    pieces = [None, None, None]
    joined = b"|".join(OPTIONS)
    while len(pieces) < count:
        r = rng.random()
        if r < 0.6:
            a = int(rng.integers(0, len(joined)))
            pieces.append(joined[a:a + int(rng.integers(1, 5))])
        elif r < 0.9:
            pieces.append(bytes(rng.integers(0, 256, size=int(rng.integers(1, 4))).tolist()))
        else:
            pieces.append(b"" if r < 0.95 else None)
    return pieces


def test_token_table_layout():
    data, offsets = token_table([b"ab", None, b"", b"c"])
    assert data.tobytes() == b"abc"
    assert offsets.tolist() == [0, 2, 2, 2, 3]


def test_mask_words_layout():
    flags = [False] * 64
    flags[0] = flags[33] = flags[63] = True
    assert og.mask_words(flags).tolist() == [1, (1 << 1) | (1 << 31)]


def test_literal_automaton_matches_literal_state():
    rng = np.random.default_rng(3)
    pieces = _pieces(rng, 700)
    for permitted in (None, [0, 1, 3], [4, 2]):
        trans, complete, start = literal_automaton(OPTIONS, permitted)
        for _ in range(25):
            machine, state = og.NameChoice(OPTIONS, permitted), start
            for _ in range(12):
                if machine.is_complete():
                    assert complete[state]
                    break
                assert not complete[state]
                want = og.allowed(pieces, machine)
                got = og.automaton_mask(trans, complete, pieces, state, CALL_END)
                assert got == want
                ids = [t for t, ok in enumerate(want) if ok]
                if not ids:
                    break
                # mostly allowed pieces; now and then a rejected one (partial advance)
                token = int(rng.choice(ids)) if rng.random() < 0.85 else int(rng.integers(3, len(pieces)))
                og.advance(pieces, machine, token)
                state = og.automaton_advance(trans, pieces, state, token, start, CALL_START, CALL_END)


def test_automaton_markers_follow_run_turn():
    rng = np.random.default_rng(4)
    pieces = _pieces(rng, 300)
    trans, complete, start = literal_automaton(OPTIONS)
    adv = lambda s, t: og.automaton_advance(trans, pieces, s, t, start, CALL_START, CALL_END)
    assert adv(0, CALL_START) == start            # generator.rs:118-119
    assert adv(0, 7) == 0                         # no machine: other ids change nothing
    assert adv(start, CALL_END) == 0              # generator.rs:120-121
    assert adv(start, CALL_START) == start        # a marker has no bytes (mask.rs:44-48)
    assert adv(5, 0xFFFFFFFF) == 5                # a sequence that was not stepped
    # state 0 allows every id; a complete state only call_end
    assert all(og.automaton_mask(trans, complete, pieces, 0, CALL_END))
    done = int(np.nonzero(complete)[0][0])
    flags = og.automaton_mask(trans, complete, pieces, done, CALL_END)
    assert [t for t, ok in enumerate(flags) if ok] == [CALL_END]
    # a piece rejected half-way keeps the bytes it had consumed (mask.rs:44-48 with all())
    s = adv(start, CALL_START) if False else start
    for t, piece in enumerate(pieces):
        if piece == b"gex":
            break
    else:
        pieces.append(b"gex")
        t = len(pieces) - 1
    m = og.NameChoice(OPTIONS)
    assert not og.advance(pieces, m, t) and m.literal.position == 2
    s = adv(s, t)
    assert og.automaton_mask(trans, complete, pieces, s, CALL_END) == og.allowed(pieces, m)
