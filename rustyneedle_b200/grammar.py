"""Device grammar masks: the host side of nb_token_automaton_*.

The reference constrains a tool call by stepping its call machine over every
vocabulary piece on the host (TokenBytes::allowed, crates/grammar/src/mask.rs:28-42)
and advancing it with the chosen piece (TokenBytes::advance, mask.rs:44-49)
inside run_turn (crates/generate/src/generator.rs:102-124). Here a machine is
compiled into a byte automaton once, and the masks and the advance run on the
device for a whole batch (`TokenAutomaton`).

`token_table` lays out the vocabulary as TokenBytes::new does (mask.rs:12-22:
a piece per id, None for ids without bytes). `literal_automaton` compiles a
Literals machine (LiteralState, crates/grammar/src/machine.rs:278-312), the
form a call's tool-name choice takes (call.rs:87-90), into a trie automaton.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._native import Model, _check, _ptr, lib


def token_table(pieces: list) -> tuple[np.ndarray, np.ndarray]:
    """(bytes uint8, offsets uint32[len(pieces) + 1]); None and b"" both give an empty range."""
    offsets = np.zeros(len(pieces) + 1, dtype=np.uint32)
    chunks = []
    total = 0
    for i, piece in enumerate(pieces):
        if piece:
            chunks.append(bytes(piece))
            total += len(piece)
        offsets[i + 1] = total
    data = np.frombuffer(b"".join(chunks), dtype=np.uint8).copy() if chunks else np.zeros(0, dtype=np.uint8)
    return data, offsets


def literal_automaton(options: list, permitted: list | None = None) -> tuple[np.ndarray, np.ndarray, int]:
    """Trie automaton of LiteralState::restricted(options, permitted) (machine.rs:290-303).

    A LiteralState is its alive options and its position; the states reachable
    from the start are exactly the prefixes shared by the alive options, so the
    trie over the permitted options' bytes is the machine. Returns
    (transitions [S][256] uint32, complete [S] uint8, start = 1); state 0 is the
    "no machine" state and every rejected byte maps to 0. complete marks a node
    that ends an option (can_finish, machine.rs:305-307) and has no longer
    option beneath it: the machine accepts no further byte.
    """
    chosen = range(len(options)) if permitted is None else permitted
    edges: list[dict] = [{}, {}]
    ends = [False, False]
    for index in chosen:
        node = 1
        for byte in bytes(options[index]):
            nxt = edges[node].get(byte)
            if nxt is None:
                nxt = len(edges)
                edges[node][byte] = nxt
                edges.append({})
                ends.append(False)
            node = nxt
        ends[node] = True
    transitions = np.zeros((len(edges), 256), dtype=np.uint32)
    complete = np.zeros(len(edges), dtype=np.uint8)
    for node, out in enumerate(edges):
        for byte, nxt in out.items():
            transitions[node, byte] = nxt
        complete[node] = 1 if (node != 0 and ends[node] and not out) else 0
    return transitions, complete, 1


def _address(buffer) -> int | None:
    """Device address of a torch tensor, or an int address as given."""
    if buffer is None:
        return None
    return int(buffer.data_ptr()) if hasattr(buffer, "data_ptr") else int(buffer)


class TokenAutomaton:
    """A compiled call machine on the model's GPU (nb_token_automaton_*)."""

    def __init__(self, model: Model, transitions: np.ndarray, complete: np.ndarray, start: int, pieces: list,
                 call_start: int, call_end: int):
        trans = np.ascontiguousarray(transitions, dtype=np.uint32)
        comp = np.ascontiguousarray(complete, dtype=np.uint8)
        if trans.ndim != 2 or trans.shape[1] != 256 or comp.shape != (trans.shape[0],):
            raise ValueError("transitions must be [states][256] and complete [states]")
        data, offsets = token_table(pieces)
        self.model = model
        self.num_states = int(trans.shape[0])
        h = ctypes.c_void_p()
        _check(lib().nb_token_automaton_create(model._h, _ptr(trans), self.num_states, _ptr(comp), int(start),
                                               _ptr(data) if data.size else None, _ptr(offsets), len(pieces),
                                               int(call_start), int(call_end), ctypes.byref(h)))
        self._h = h

    def mask(self, states, mask_bits, count: int | None = None) -> None:
        """Device mask words [count][vocab/32] for device states (uint32/int32 tensors)."""
        n = int(states.numel()) if count is None else count
        _check(lib().nb_token_automaton_mask(self._h, _address(states), n, _address(mask_bits)))

    def advance(self, next_ids, states, count: int | None = None) -> None:
        n = int(states.numel()) if count is None else count
        _check(lib().nb_token_automaton_advance(self._h, _address(next_ids), n, _address(states)))

    def check(self) -> None:
        _check(lib().nb_token_automaton_check(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nb_token_automaton_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
