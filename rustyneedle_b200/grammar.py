"""Device grammar masks: the host side of nb_token_automaton_*.

The reference constrains a tool call by stepping its call machine over every
vocabulary piece on the host (TokenBytes::allowed, crates/grammar/src/mask.rs:28-42)
and advancing it with the chosen piece (TokenBytes::advance, mask.rs:44-49)
inside run_turn (crates/generate/src/generator.rs:102-124). Here a machine is
compiled into a byte automaton once, and the masks and the advance run on the
device for a whole batch (`TokenAutomaton`).

`token_table` lays out the vocabulary as TokenBytes::new does (mask.rs:12-22:
a piece per id, None for ids without bytes). `call_automaton` compiles a whole
tool-call grammar — CallGrammar::from_tools_json and its CallMachine
(crates/grammar/src/call.rs:16-174, every schema form of schema.rs and
machine.rs) — in the library (nb_call_grammar_compile, host only).
`literal_automaton` compiles a tool-name choice alone (the Name stage of
CallMachine::step, call.rs:123-130) into a trie automaton.
"""
from __future__ import annotations

import ctypes
import json

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
    """Trie automaton of the Name stage of CallMachine::step (call.rs:123-130)
    over LiteralState::restricted(options, permitted) (machine.rs:290-312).

    A LiteralState is its alive options and its position; the states reachable
    from the start are the prefixes the alive options share, so the trie of the
    permitted options is the machine. The stage ends as soon as chosen() finds
    an alive option that has ended, so a node that ends an option is complete
    and nothing beneath it is reachable (with 'get' and 'get_user' permitted,
    'get' is chosen after its third byte). Returns (transitions [S][256]
    uint32, complete [S] uint8, start = 1); state 0 is the "no machine" state
    and every rejected byte maps to 0.
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
    # keep what the stage can reach: nothing below a node that ends an option
    number = {1: 1}
    order = [1]
    for node in order:
        if ends[node]:
            continue
        for byte, nxt in sorted(edges[node].items()):
            number[nxt] = len(order) + 1
            order.append(nxt)
    transitions = np.zeros((len(order) + 1, 256), dtype=np.uint32)
    complete = np.zeros(len(order) + 1, dtype=np.uint8)
    for node in order:
        s = number[node]
        complete[s] = 1 if ends[node] else 0
        if not ends[node]:
            for byte, nxt in edges[node].items():
                transitions[s, byte] = number[nxt]
    return transitions, complete, 1


def call_automaton(tools, require_call: bool = False, permitted: list | None = None,
                   max_states: int = 0) -> tuple[np.ndarray, np.ndarray, int]:
    """The byte automaton of CallGrammar::from_tools_json(tools) (call.rs:47-49),
    with require_call(permitted) when require_call (call.rs:51-55), compiled by
    the library on the host (nb_call_grammar_compile). `tools` is the JSON text
    or the decoded list. Returns (transitions [S][256] uint32, complete [S]
    uint8, start), the tables TokenAutomaton takes. Raises NeedleError with
    NB_ERR_UNSUPPORTED when the machine has more than max_states states."""
    text = tools if isinstance(tools, str) else json.dumps(tools)
    L = lib()
    if not getattr(L, "_call_grammar_declared", False):
        P, U32 = ctypes.c_void_p, ctypes.c_uint32
        L.nb_call_grammar_compile.argtypes = [ctypes.c_char_p, ctypes.c_int, P, ctypes.c_size_t, U32, ctypes.POINTER(P)]
        L.nb_call_grammar_compile.restype = ctypes.c_int
        L.nb_call_grammar_states.argtypes = [P]
        L.nb_call_grammar_states.restype = U32
        L.nb_call_grammar_tables.argtypes = [P, P, P, ctypes.POINTER(U32)]
        L.nb_call_grammar_tables.restype = ctypes.c_int
        L.nb_call_grammar_release.argtypes = [P]
        L.nb_call_grammar_release.restype = None
        L._call_grammar_declared = True
    allowed = None if permitted is None else np.ascontiguousarray(permitted, dtype=np.uint32)
    h = ctypes.c_void_p()
    _check(L.nb_call_grammar_compile(text.encode(), 1 if require_call else 0,
                                     _ptr(allowed) if allowed is not None and allowed.size else None,
                                     0 if allowed is None else allowed.size, max_states, ctypes.byref(h)))
    try:
        n = int(L.nb_call_grammar_states(h))
        transitions = np.zeros((n, 256), dtype=np.uint32)
        complete = np.zeros(n, dtype=np.uint8)
        start = ctypes.c_uint32()
        _check(L.nb_call_grammar_tables(h, _ptr(transitions), _ptr(complete), ctypes.byref(start)))
    finally:
        L.nb_call_grammar_release(h)
    return transitions, complete, int(start.value)


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

    # The kernels run on the model's CUDA stream. Buffers that torch has just
    # written on its own stream must be complete before they are read there,
    # and torch must not read the results before the model's stream is done:
    # with sync (the default) the wrapper waits for torch's current stream
    # before queuing and for the model's stream after it.
    def _torch_ready(self, *buffers) -> None:
        for b in buffers:
            if hasattr(b, "data_ptr") and getattr(b, "is_cuda", False):
                import torch

                torch.cuda.current_stream(b.device).synchronize()
                return

    def mask(self, states, mask_bits, count: int | None = None, sync: bool = True) -> None:
        """Device mask words [count][vocab/32] for device states (uint32/int32 tensors)."""
        n = int(states.numel()) if count is None else count
        if sync:
            self._torch_ready(states, mask_bits)
        _check(lib().nb_token_automaton_mask(self._h, _address(states), n, _address(mask_bits)))
        if sync:
            self.model.synchronize()

    def advance(self, next_ids, states, count: int | None = None, sync: bool = True) -> None:
        """Advances the device states with the chosen ids (run_turn's markers included)."""
        n = int(states.numel()) if count is None else count
        if sync:
            self._torch_ready(next_ids, states)
        _check(lib().nb_token_automaton_advance(self._h, _address(next_ids), n, _address(states)))
        if sync:
            self.model.synchronize()

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
