"""CPU restatement of the reference's grammar mask step — TEST INFRASTRUCTURE.

Only tests/ and bench.py's CPU baseline use this module, as the checker of the
device token automaton; nothing in the product imports it.

  LiteralMachine      LiteralState (crates/grammar/src/machine.rs:278-312) and
                      its restricted form (290-292)
  allowed / advance   TokenBytes::allowed / advance (crates/grammar/src/mask.rs:28-49),
                      including allowed's per-first-byte cache
  run_turn_choice     the constrained branch of run_turn (generator.rs:102-124):
                      complete → call_end; else mask; markers enter/leave the machine
  automaton_mask / automaton_advance
                      the same two operations over a byte automaton (0 = rejected,
                      state 0 = no machine), the form the device kernels take
"""
from __future__ import annotations

import numpy as np


class LiteralMachine:
    """LiteralState: alive option indices and a byte position (machine.rs:278-312)."""

    def __init__(self, options: list, allowed: list | None = None):
        self.options = [bytes(o) for o in options]
        self.alive = list(range(len(options))) if allowed is None else list(allowed)
        self.position = 0

    def clone(self) -> "LiteralMachine":
        other = LiteralMachine.__new__(LiteralMachine)
        other.options, other.alive, other.position = self.options, list(self.alive), self.position
        return other

    def step(self, byte: int) -> bool:
        # machine.rs:294-303: survivors hold `byte` at `position`; none → reject, state kept
        survivors = [i for i in self.alive
                     if self.position < len(self.options[i]) and self.options[i][self.position] == byte]
        if not survivors:
            return False
        self.alive = survivors
        self.position += 1
        return True

    def can_finish(self) -> bool:
        return any(len(self.options[i]) == self.position for i in self.alive)

    def accepts_more(self) -> bool:
        return any(len(self.options[i]) > self.position for i in self.alive)


def allowed(pieces: list, machine) -> list:
    """TokenBytes::allowed (mask.rs:28-42)."""
    first_ok: dict = {}
    out = []
    for piece in pieces:
        if not piece:
            out.append(False)
            continue
        first = piece[0]
        if first not in first_ok:
            first_ok[first] = machine.clone().step(first)
        if not first_ok[first]:
            out.append(False)
            continue
        trial = machine.clone()
        out.append(all(trial.step(b) for b in piece))
    return out


def advance(pieces: list, machine, token: int) -> bool:
    """TokenBytes::advance (mask.rs:44-49): steps until the first rejected byte."""
    piece = pieces[token] if 0 <= token < len(pieces) else None
    if piece is None:
        return False
    return all(machine.step(b) for b in piece)


def mask_words(flags) -> np.ndarray:
    """Bit t of word t // 32 set where flags[t] (the boundary's mask layout)."""
    bits = np.asarray(flags, dtype=bool)
    pad = (-bits.size) % 32
    bits = np.concatenate([bits, np.zeros(pad, dtype=bool)]).reshape(-1, 32)
    return (bits.astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(axis=1).astype(np.uint32)


def automaton_mask(transitions: np.ndarray, complete: np.ndarray, pieces: list, state: int, call_end: int) -> list:
    """One sequence's allowed ids over a byte automaton."""
    V = len(pieces)
    if state == 0:
        return [True] * V
    if complete[state]:
        return [t == call_end for t in range(V)]
    out = []
    for piece in pieces:
        q = state
        if not piece:
            out.append(False)
            continue
        for b in piece:
            q = int(transitions[q, b])
            if q == 0:
                break
        out.append(q != 0)
    return out


def automaton_advance(transitions: np.ndarray, pieces: list, state: int, token: int, start: int, call_start: int,
                      call_end: int) -> int:
    """generator.rs:118-124 over a byte automaton; the last accepted state is kept."""
    if token == 0xFFFFFFFF:
        return state
    if token == call_start and state == 0:
        return start
    if token == call_end:
        return 0
    if state != 0 and 0 <= token < len(pieces) and pieces[token]:
        for b in pieces[token]:
            q = int(transitions[state, b])
            if q == 0:
                break
            state = q
    return state
