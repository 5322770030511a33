"""ctypes binding of include/needle_b200.h (the product's C ABI)."""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# $NEEDLE_B200_LIBRARY selects another build of the library (same ABI)
_LIBRARY = os.environ.get("NEEDLE_B200_LIBRARY") or os.path.join(HERE, "_native", "libneedle_b200.so")

NB_OK = 0
STATUS_NAMES = {
    -1: "NB_ERR_IO", -2: "NB_ERR_ARCHIVE", -3: "NB_ERR_DEPTH", -4: "NB_ERR_ARGUMENT", -5: "NB_ERR_UNSUPPORTED",
    -6: "NB_ERR_CUDA", -7: "NB_ERR_CONTEXT_OVERFLOW", -8: "NB_ERR_KV_EXHAUSTED", -9: "NB_ERR_TIMEOUT",
    -10: "NB_ERR_NO_DEVICE",
}


class NeedleError(RuntimeError):
    """A failed C-ABI call; `status` is the nb_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class DepthError(NeedleError):
    """ModelError::Depth (crates/model/src/model.rs:15)."""


class ContextOverflow(NeedleError):
    """The session would pass max_seq_len (crates/generate/src/generator.rs:77-89)."""


class nb_options(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("max_sessions", ctypes.c_uint32), ("kv_pages", ctypes.c_uint32),
                ("max_batch_tokens", ctypes.c_uint32)]


class nb_model_config(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint32) for name in
                ("vocab", "output_vocab", "d_model", "num_heads", "num_kv_heads", "num_layers", "head_dim",
                 "max_seq_len", "hada_n", "lanes", "depth")] + [("active_layers", ctypes.c_int32 * 64),
                                                               ("rope_theta", ctypes.c_float)]


class nb_step_stats(ctypes.Structure):
    _fields_ = [("probability", ctypes.c_float), ("mass", ctypes.c_float), ("status", ctypes.c_int32)]


_lib = None


def library_path() -> str:
    return _LIBRARY


def lib() -> ctypes.CDLL:
    """The loaded native library; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIBRARY):
            raise ImportError(f"{_LIBRARY} is missing: run `python -m rustyneedle_b200.build` "
                              "(or __graft_entry__.build()) first; there is no CPU fallback")
        L = ctypes.CDLL(_LIBRARY)
        P, U32, SZ, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_int
        sig = {
            "nb_last_error": (ctypes.c_char_p, []),
            "nb_model_open": (I, [ctypes.c_char_p, ctypes.POINTER(nb_options), ctypes.POINTER(P)]),
            "nb_model_with_depth": (I, [P, U32, ctypes.POINTER(P)]),
            "nb_model_get_config": (I, [P, ctypes.POINTER(nb_model_config)]),
            "nb_model_release": (None, [P]),
            "nb_model_synchronize": (I, [P]),
            "nb_session_create": (I, [P, ctypes.POINTER(P)]),
            "nb_session_clone": (I, [P, ctypes.POINTER(P)]),
            "nb_session_release": (None, [P]),
            "nb_session_feed": (I, [P, P, SZ]),
            "nb_sessions_feed": (I, [P, P, P, SZ]),
            "nb_session_push": (I, [P, U32]),
            "nb_session_logits": (I, [P, P, SZ]),
            "nb_cross_memory_create": (I, [P, P, SZ, P]),
            "nb_cross_memory_release": (None, [P]),
            "nb_session_set_cross": (I, [P, P]),
            "nb_model_text_vocab": (SZ, [P]),
            "nb_session_head_output": (I, [P, U32, P, SZ, ctypes.POINTER(SZ)]),
            "nb_session_pooled_readout": (I, [P, U32, P, SZ, ctypes.POINTER(SZ)]),
            "nb_session_len": (SZ, [P]),
            "nb_session_step": (I, [P, P, ctypes.POINTER(U32), ctypes.POINTER(nb_step_stats)]),
            "nb_batch_create": (I, [P, P, U32, ctypes.POINTER(P)]),
            "nb_batch_release": (None, [P]),
            "nb_batch_step": (I, [P, P, P, P]),
            "nb_batch_step_device": (I, [P, P, P, P]),
            "nb_batch_run": (I, [P, U32, P, P, ctypes.POINTER(ctypes.c_float)]),
            "nb_build_expf_table": (I, [ctypes.c_char_p]),
            "nb_token_automaton_create": (I, [P, P, U32, P, U32, P, P, U32, U32, U32, ctypes.POINTER(P)]),
            "nb_token_automaton_release": (None, [P]),
            "nb_token_automaton_mask": (I, [P, P, U32, P]),
            "nb_token_automaton_advance": (I, [P, P, U32, P]),
            "nb_token_automaton_check": (I, [P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != NB_OK:
        message = lib().nb_last_error().decode(errors="replace")
        cls = DepthError if status == -3 else ContextOverflow if status == -7 else NeedleError
        raise cls(status, message)


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


@dataclass
class ModelConfig:
    vocab: int
    output_vocab: int
    d_model: int
    num_heads: int
    num_kv_heads: int
    num_layers: int
    head_dim: int
    max_seq_len: int
    hada_n: int
    lanes: int
    active_layers: list
    rope_theta: float


@dataclass
class StepStats:
    probability: float
    mass: float
    status: int


class Model:
    """Model::open / Model::with_depth. Handles share one set of device weights."""

    def __init__(self, handle):
        self._h = handle
        c = nb_model_config()
        _check(lib().nb_model_get_config(self._h, ctypes.byref(c)))
        self.config = ModelConfig(c.vocab, c.output_vocab, c.d_model, c.num_heads, c.num_kv_heads, c.num_layers,
                                  c.head_dim, c.max_seq_len, c.hada_n, c.lanes, list(c.active_layers[:c.depth]),
                                  c.rope_theta)

    @classmethod
    def open(cls, path: str, device: int = -1, max_sessions: int = 0, kv_pages: int = 0,
             max_batch_tokens: int = 0) -> "Model":
        h = ctypes.c_void_p()
        opts = nb_options(device, max_sessions, kv_pages, max_batch_tokens)
        _check(lib().nb_model_open(os.fspath(path).encode(), ctypes.byref(opts), ctypes.byref(h)))
        return cls(h)

    def with_depth(self, depth: int) -> "Model":
        h = ctypes.c_void_p()
        _check(lib().nb_model_with_depth(self._h, depth, ctypes.byref(h)))
        return Model(h)

    def active_layers(self) -> list:
        return list(self.config.active_layers)

    def text_vocab(self) -> int:
        """AudioManifest::text_vocab of a Whistle archive (0 without an audio section)."""
        return int(lib().nb_model_text_vocab(self._h))

    def synchronize(self) -> None:
        _check(lib().nb_model_synchronize(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nb_model_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """Session::new / feed / push / logits / len, plus Clone."""

    def __init__(self, model: Model, handle=None):
        self.model = model
        if handle is None:
            handle = ctypes.c_void_p()
            _check(lib().nb_session_create(model._h, ctypes.byref(handle)))
        self._h = handle

    def clone(self) -> "Session":
        h = ctypes.c_void_p()
        _check(lib().nb_session_clone(self._h, ctypes.byref(h)))
        return Session(self.model, h)

    def __len__(self) -> int:
        return int(lib().nb_session_len(self._h))

    def feed(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        _check(lib().nb_session_feed(self._h, _ptr(t), t.size))

    def push(self, token: int) -> None:
        _check(lib().nb_session_push(self._h, int(token)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.model.config.output_vocab, dtype=np.float32)
        _check(lib().nb_session_logits(self._h, _ptr(out), out.size))
        return out

    def set_cross(self, memory: "CrossMemory | None") -> None:
        """Every later pass attends to `memory` after each layer's attention
        (Session::push_with with a CrossState); None detaches."""
        _check(lib().nb_session_set_cross(self._h, memory._h if memory is not None else None))
        self.cross = memory

    def _head(self, fn, code: int):
        out = np.empty(1 << 14, dtype=np.float32)
        n = ctypes.c_size_t()
        status = fn(self._h, int(code), _ptr(out), out.size, ctypes.byref(n))
        if status == -4:  # NB_ERR_ARGUMENT: the model has no head with that code (the reference's None)
            return None
        _check(status)
        return out[:n.value].copy()

    def head_output(self, code: int):
        """Session::head_output: the probe head's projection, or None without that head."""
        return self._head(lib().nb_session_head_output, code)

    def pooled_readout(self, code: int):
        """Session::pooled_readout: the head's pooled readout, or None without that head."""
        return self._head(lib().nb_session_pooled_readout, code)

    def step(self, mask_bits: np.ndarray | None = None, stats: bool = False):
        """One greedy step: choose from the current logits (optionally under a
        packed allowed-token bitset), push the choice, return it."""
        nxt = ctypes.c_uint32()
        st = nb_step_stats()
        m = None if mask_bits is None else np.ascontiguousarray(mask_bits, dtype=np.uint32)
        _check(lib().nb_session_step(self._h, None if m is None else _ptr(m), ctypes.byref(nxt),
                                     ctypes.byref(st) if stats else None))
        if stats:
            return int(nxt.value), StepStats(st.probability, st.mass, st.status)
        return int(nxt.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nb_session_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CrossMemory:
    """CrossWeights::memory of an encoder output [frames][d_model] (Whistle)."""

    def __init__(self, model: Model, encoded: np.ndarray):
        enc = np.ascontiguousarray(encoded, dtype=np.float32)
        self.model = model
        self.frames = int(enc.shape[0])
        h = ctypes.c_void_p()
        _check(lib().nb_cross_memory_create(model._h, _ptr(enc), self.frames, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nb_cross_memory_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def feed_many(sessions, prompts) -> None:
    """Feeds every session its prompt in shared forward passes (nb_sessions_feed);
    each session ends as if fed alone."""
    sessions = list(sessions)
    if len(sessions) != len(prompts):
        raise ValueError("one prompt per session")
    if not sessions:
        return
    arrays = [np.ascontiguousarray(p, dtype=np.uint32) for p in prompts]
    n = len(sessions)
    handles = (ctypes.c_void_p * n)(*[s._h for s in sessions])
    ids = (ctypes.c_void_p * n)(*[a.ctypes.data if a.size else None for a in arrays])
    counts = (ctypes.c_size_t * n)(*[a.size for a in arrays])
    _check(lib().nb_sessions_feed(handles, ids, counts, n))


class Batch:
    """B sessions stepped together by one graph-captured device step."""

    def __init__(self, model: Model, sessions: list):
        self.model = model
        self.sessions = list(sessions)
        arr = (ctypes.c_void_p * len(sessions))(*[s._h.value if isinstance(s._h, ctypes.c_void_p) else s._h
                                                   for s in sessions])
        self._arr = arr
        h = ctypes.c_void_p()
        _check(lib().nb_batch_create(model._h, ctypes.cast(arr, ctypes.c_void_p), len(sessions), ctypes.byref(h)))
        self._h = h
        self._next = np.zeros(len(sessions), dtype=np.uint32)
        self._stats = (nb_step_stats * len(sessions))()

    def step(self, mask_bits: np.ndarray | None = None, stats: bool = False):
        m = None if mask_bits is None else np.ascontiguousarray(mask_bits, dtype=np.uint32)
        if m is not None and m.size != len(self.sessions) * (self.model.config.output_vocab // 32):
            raise ValueError("mask_bits must hold count x output_vocab/32 words")
        _check(lib().nb_batch_step(self._h, None if m is None else _ptr(m), _ptr(self._next),
                                   ctypes.cast(self._stats, ctypes.c_void_p) if stats else None))
        if stats:
            return self._next.copy(), [StepStats(s.probability, s.mass, s.status) for s in self._stats]
        return self._next.copy()

    def step_device(self, mask_bits_device: int | None, next_device: int) -> None:
        """One step with device mask words (or None) and device output ids (nb_batch_step_device)."""
        _check(lib().nb_batch_step_device(self._h, mask_bits_device, next_device, None))

    def run(self, steps: int, mask_bits_device: int | None = None, tokens_device: int | None = None) -> float:
        """`steps` device-resident greedy steps; returns their device time in ms."""
        ms = ctypes.c_float()
        _check(lib().nb_batch_run(self._h, steps, mask_bits_device, tokens_device, ctypes.byref(ms)))
        return float(ms.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nb_batch_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
