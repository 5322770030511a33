"""ctypes binding of the CPU restatement in needle_oracle.cpp.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, always as the checker or the timed
CPU baseline, never as part of the product path.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "_build", "libneedle_oracle.so")

MODE_INT = 0
MODE_FLOAT = 1

_lib = None


def build() -> str:
    """Compiles the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY):
            build()
        _lib = ctypes.CDLL(LIBRARY)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    P, I, U32, SZ, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_float
    fp = ctypes.POINTER(ctypes.c_float)
    sig = {
        "nbo_last_error": (ctypes.c_char_p, []),
        "nbo_model_open": (I, [ctypes.c_char_p, I, I, ctypes.POINTER(P)]),
        "nbo_model_with_depth": (I, [P, I, ctypes.POINTER(P)]),
        "nbo_model_free": (None, [P]),
        "nbo_model_active_layers": (I, [P, P, I]),
        "nbo_model_geometry": (None, [P, P]),
        "nbo_model_set_threads": (None, [P, I]),
        "nbo_session_new": (P, [P]),
        "nbo_session_clone": (P, [P]),
        "nbo_session_free": (None, [P]),
        "nbo_session_len": (SZ, [P]),
        "nbo_session_head_output": (ctypes.c_long, [P, ctypes.c_int, P, SZ]),
        "nbo_cross_memory_new": (I, [P, P, SZ, P]),
        "nbo_cross_memory_free": (None, [P]),
        "nbo_cross_memory_read": (SZ, [P, I, P, P, P, P]),
        "nbo_session_push_cross": (I, [P, ctypes.c_uint32, P]),
        "nbo_model_text_vocab": (SZ, [P]),
        "nbo_session_pooled_readout": (ctypes.c_long, [P, ctypes.c_int, P, SZ]),
        "nbo_session_push": (None, [P, U32]),
        "nbo_session_push_traced": (None, [P, U32, P]),
        "nbo_session_feed": (None, [P, P, SZ]),
        "nbo_session_logits": (None, [P, P]),
        "nbo_session_hidden": (None, [P, P]),
        "nbo_session_cache": (SZ, [P, I, P, P, P, P]),
        "nbo_sessions_step": (None, [P, SZ, P, P, I]),
        "nbo_argmax": (ctypes.c_int32, [P, SZ]),
        "nbo_argmax_allowed": (ctypes.c_int32, [P, P, SZ]),
        "nbo_allowed_statistics": (None, [P, SZ, U32, P, fp, fp]),
        "nbo_walsh": (None, [P, SZ]),
        "nbo_fast_exp": (F, [F]),
        "nbo_sigmoid": (F, [F]),
        "nbo_softmax": (None, [P, SZ]),
        "nbo_kronecker": (None, [P, P, SZ, P, SZ, P, I]),
        "nbo_sinkhorn": (None, [P, SZ, SZ]),
        "nbo_zero_centred_norm": (None, [P, P, P, SZ]),
        "nbo_fake_quantise_int8": (None, [P, SZ]),
        "nbo_quantise_int8": (F, [P, P, SZ]),
        "nbo_rotary": (None, [P, SZ, SZ, F]),
        "nbo_ladder_order": (I, [I, P]),
        "nbo_ladder_select": (I, [I, I, P]),
        "nbo_half_to_f32": (F, [ctypes.c_uint16]),
        "nbo_matrix_product": (I, [P, I, P, SZ, SZ, P, P]),
        "nbo_matrix_dequantise_row": (I, [P, I, SZ, P]),
        "nbo_product_raw": (I, [I, U32, P, P, P, SZ, SZ, P, P, P]),
        "nbo_tensor_info": (I, [P, I, P]),
        "nbo_hadamard_apply": (I, [P, I, P, P]),
        "nbo_attend_head_raw": (I, [I, P, F, P, P, P, P, SZ, SZ, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


class OracleError(RuntimeError):
    def __init__(self, status: int):
        super().__init__(f"oracle status {status}: {lib().nbo_last_error().decode()}")
        self.status = status


class Model:
    """Model::open / with_depth of the CPU restatement."""

    def __init__(self, handle, mode: int):
        self._h = handle
        self.mode = mode
        g = np.zeros(8, dtype=np.int32)
        lib().nbo_model_geometry(self._h, _ptr(g))
        (self.vocab, self.output_vocab, self.d_model, self.num_heads, self.num_kv_heads, self.num_layers,
         self.head_dim, self.max_seq_len) = (int(x) for x in g)

    @classmethod
    def open(cls, path: str, mode: int = MODE_INT, threads: int = 1) -> "Model":
        h = ctypes.c_void_p()
        status = lib().nbo_model_open(path.encode(), mode, threads, ctypes.byref(h))
        if status:
            raise OracleError(status)
        return cls(h, mode)

    def with_depth(self, depth: int) -> "Model":
        h = ctypes.c_void_p()
        status = lib().nbo_model_with_depth(self._h, depth, ctypes.byref(h))
        if status:
            raise OracleError(status)
        return Model(h, self.mode)

    def set_threads(self, threads: int) -> None:
        lib().nbo_model_set_threads(self._h, threads)

    def active_layers(self) -> list[int]:
        out = np.zeros(64, dtype=np.int32)
        n = lib().nbo_model_active_layers(self._h, _ptr(out), 64)
        return [int(x) for x in out[:n]]

    def matrix_product(self, tensor: int, x: np.ndarray, first_row: int = 0, rows: int | None = None):
        info = self.tensor_info(tensor)
        rows = info["rows"] - first_row if rows is None else rows
        groups = -(-info["columns"] // info["group"])
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(rows, dtype=np.float32)
        sums = np.zeros((rows, groups), dtype=np.int32)
        status = lib().nbo_matrix_product(self._h, tensor, _ptr(x), first_row, rows, _ptr(out), _ptr(sums))
        if status:
            raise OracleError(status)
        return out, sums

    def dequantise_row(self, tensor: int, row: int) -> np.ndarray:
        info = self.tensor_info(tensor)
        out = np.zeros(info["columns"], dtype=np.float32)
        status = lib().nbo_matrix_dequantise_row(self._h, tensor, row, _ptr(out))
        if status:
            raise OracleError(status)
        return out

    def tensor_info(self, tensor: int) -> dict:
        o = np.zeros(5, dtype=np.int64)
        if lib().nbo_tensor_info(self._h, tensor, _ptr(o)):
            raise OracleError(-4)
        return dict(kind=int(o[0]), rows=int(o[1]), columns=int(o[2]), group=int(o[3]), bits=int(o[4]))

    def hadamard(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(self.d_model, dtype=np.float32)
        status = lib().nbo_hadamard_apply(self._h, layer, _ptr(x), _ptr(out))
        if status:
            raise OracleError(status)
        return out

    def route(self, layer: int, slot: int, stream: np.ndarray):
        """LaneWeights::route: (block input [d], post gates [lanes], residual mixing [lanes·lanes])."""
        s = np.ascontiguousarray(stream, dtype=np.float32)
        lanes = s.size // self.d_model
        block_input = np.zeros(self.d_model, dtype=np.float32)
        post = np.zeros(lanes, dtype=np.float32)
        residual = np.zeros(lanes * lanes, dtype=np.float32)
        status = lib().nbo_route(self._h, layer, slot, _ptr(s), _ptr(block_input), _ptr(post), _ptr(residual))
        if status:
            raise OracleError(status)
        return block_input, post, residual

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.nbo_model_free(self._h)
            self._h = None


class Session:
    def __init__(self, model: Model, handle=None):
        self.model = model
        self._h = handle if handle is not None else lib().nbo_session_new(model._h)

    def clone(self) -> "Session":
        return Session(self.model, lib().nbo_session_clone(self._h))

    def __len__(self) -> int:
        return int(lib().nbo_session_len(self._h))

    def _head(self, fn, code: int):
        out = np.empty(1 << 14, dtype=np.float32)
        n = fn(self._h, int(code), _ptr(out), out.size)
        return None if n < 0 else out[:n].copy()

    def push_cross(self, token: int, memory: "CrossMemory") -> None:
        """Session::push_with(token, CrossState) (whistle lib.rs:255-293)."""
        status = lib().nbo_session_push_cross(self._h, int(token), memory._h)
        if status:
            raise OracleError(status)

    def head_output(self, code: int):
        """Session::head_output (session.rs:150-154); None without that head."""
        return self._head(lib().nbo_session_head_output, code)

    def pooled_readout(self, code: int):
        """Session::pooled_readout (session.rs:156-160); None without that head."""
        return self._head(lib().nbo_session_pooled_readout, code)

    def push(self, token: int) -> None:
        lib().nbo_session_push(self._h, int(token))

    def push_traced(self, token: int) -> np.ndarray:
        depth = len(self.model.active_layers())
        trace = np.zeros((depth, 4, self.model.d_model), dtype=np.float32)
        lib().nbo_session_push_traced(self._h, int(token), _ptr(trace))
        return trace

    def feed(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        lib().nbo_session_feed(self._h, _ptr(t), t.size)

    def logits(self) -> np.ndarray:
        out = np.zeros(self.model.output_vocab, dtype=np.float32)
        lib().nbo_session_logits(self._h, _ptr(out))
        return out

    def hidden(self) -> np.ndarray:
        out = np.zeros(self.model.d_model, dtype=np.float32)
        lib().nbo_session_hidden(self._h, _ptr(out))
        return out

    def cache(self, layer: int):
        m = self.model
        n = len(self)
        keys = np.zeros((n, m.num_kv_heads, m.head_dim), dtype=np.int8)
        values = np.zeros_like(keys)
        ks = np.zeros((m.num_kv_heads, n), dtype=np.float32)
        vs = np.zeros_like(ks)
        count = lib().nbo_session_cache(self._h, layer, _ptr(keys), _ptr(ks), _ptr(values), _ptr(vs))
        return keys[:count], ks[:, :count], values[:count], vs[:, :count]

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.nbo_session_free(self._h)
            self._h = None


def sessions_step(sessions: list[Session], tokens, threads: int = 0, want_logits: bool = True):
    handles = (ctypes.c_void_p * len(sessions))(*[s._h for s in sessions])
    t = np.ascontiguousarray(tokens, dtype=np.uint32)
    vocab = sessions[0].model.output_vocab
    out = np.zeros((len(sessions), vocab), dtype=np.float32) if want_logits else None
    lib().nbo_sessions_step(handles, len(sessions), _ptr(t), _ptr(out) if out is not None else None, threads)
    return out


def product_raw(mode: int, bits: int, packed: np.ndarray, levels: np.ndarray, norms: np.ndarray, rows: int, cols: int,
                x: np.ndarray) -> np.ndarray:
    """A codebook product through a matrix in the archive's representation
    (packed indices, levels, fp16 norms as uint16) for one input row."""
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    lv = np.ascontiguousarray(levels, dtype=np.float32)
    nm = np.ascontiguousarray(norms, dtype=np.uint16)
    xv = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(rows, dtype=np.float32)
    status = lib().nbo_product_raw(mode, bits, _ptr(p), _ptr(lv), _ptr(nm), rows, cols, _ptr(xv), _ptr(out), None)
    if status != 0:
        raise RuntimeError(lib().nbo_last_error().decode())
    return out


def attend_head_raw(mode: int, query: np.ndarray, query_scale: float, keys: np.ndarray, key_scales: np.ndarray,
                    values: np.ndarray, value_scales: np.ndarray) -> np.ndarray:
    """One head's attention over positions given directly (keys, values
    [count][dim] int8; their scales [count])."""
    q = np.ascontiguousarray(query, dtype=np.int8)
    k = np.ascontiguousarray(keys, dtype=np.int8)
    v = np.ascontiguousarray(values, dtype=np.int8)
    ks = np.ascontiguousarray(key_scales, dtype=np.float32)
    vs = np.ascontiguousarray(value_scales, dtype=np.float32)
    count, dim = k.shape
    out = np.zeros(dim, dtype=np.float32)
    status = lib().nbo_attend_head_raw(mode, _ptr(q), float(query_scale), _ptr(k), _ptr(ks), _ptr(v), _ptr(vs), count, dim, _ptr(out))
    if status != 0:
        raise RuntimeError(lib().nbo_last_error().decode())
    return out


def argmax(values: np.ndarray) -> int:
    v = np.ascontiguousarray(values, dtype=np.float32)
    return int(lib().nbo_argmax(_ptr(v), v.size))


def argmax_allowed(values: np.ndarray, allowed: np.ndarray) -> int:
    v = np.ascontiguousarray(values, dtype=np.float32)
    a = np.ascontiguousarray(allowed, dtype=np.uint8)
    return int(lib().nbo_argmax_allowed(_ptr(v), _ptr(a), v.size))


def allowed_statistics(logits: np.ndarray, token: int, allowed: np.ndarray):
    v = np.ascontiguousarray(logits, dtype=np.float32)
    a = np.ascontiguousarray(allowed, dtype=np.uint8)
    p, m = ctypes.c_float(), ctypes.c_float()
    lib().nbo_allowed_statistics(_ptr(v), v.size, int(token), _ptr(a), ctypes.byref(p), ctypes.byref(m))
    return p.value, m.value


def walsh(values: np.ndarray) -> np.ndarray:
    v = np.array(values, dtype=np.float32)
    lib().nbo_walsh(_ptr(v), v.size)
    return v


def fast_exp(x: float) -> float:
    return float(lib().nbo_fast_exp(float(x)))


def sigmoid(x: float) -> float:
    return float(lib().nbo_sigmoid(float(x)))


def softmax(values: np.ndarray) -> np.ndarray:
    v = np.array(values, dtype=np.float32)
    lib().nbo_softmax(_ptr(v), v.size)
    return v


def kronecker(x: np.ndarray, left: np.ndarray, right: np.ndarray, mode: int = MODE_FLOAT) -> np.ndarray:
    x, left, right = (np.ascontiguousarray(a, dtype=np.float32) for a in (x, left, right))
    ls, rs = int(round(left.size ** 0.5)), int(round(right.size ** 0.5))
    out = np.zeros(ls * rs, dtype=np.float32)
    lib().nbo_kronecker(_ptr(x), _ptr(left), ls, _ptr(right), rs, _ptr(out), mode)
    return out


def sinkhorn(logits: np.ndarray, size: int, iterations: int = 20) -> np.ndarray:
    v = np.array(logits, dtype=np.float32)
    lib().nbo_sinkhorn(_ptr(v), size, iterations)
    return v


def zero_centred_norm(x: np.ndarray, gains: np.ndarray) -> np.ndarray:
    x, gains = (np.ascontiguousarray(a, dtype=np.float32) for a in (x, gains))
    out = np.zeros_like(x)
    lib().nbo_zero_centred_norm(_ptr(x), _ptr(gains), _ptr(out), x.size)
    return out


def fake_quantise_int8(x: np.ndarray) -> np.ndarray:
    v = np.array(x, dtype=np.float32)
    lib().nbo_fake_quantise_int8(_ptr(v), v.size)
    return v


def quantise_int8(x: np.ndarray):
    v = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(v.size, dtype=np.int8)
    scale = lib().nbo_quantise_int8(_ptr(v), _ptr(codes), v.size)
    return codes, float(scale)


def rotary(head: np.ndarray, position: int, theta: float = 10000.0) -> np.ndarray:
    v = np.array(head, dtype=np.float32)
    lib().nbo_rotary(_ptr(v), v.size, position, theta)
    return v


def ladder_order(layers: int) -> list[int]:
    out = np.zeros(max(layers, 1), dtype=np.int32)
    n = lib().nbo_ladder_order(layers, _ptr(out))
    return [int(x) for x in out[:n]]


def ladder_select(layers: int, depth: int):
    out = np.zeros(max(layers, 1), dtype=np.int32)
    n = lib().nbo_ladder_select(layers, depth, _ptr(out))
    return None if n < 0 else [int(x) for x in out[:n]]


def half_to_f32(bits: int) -> float:
    return float(lib().nbo_half_to_f32(bits))


class CrossMemory:
    """CrossWeights::memory (whistle/src/cross.rs:58-99) of an encoder output [frames][d_model]."""

    def __init__(self, model: Model, encoded: np.ndarray):
        enc = np.ascontiguousarray(encoded, dtype=np.float32)
        self.frames = enc.shape[0]
        self.model = model
        h = ctypes.c_void_p()
        status = lib().nbo_cross_memory_new(model._h, _ptr(enc), self.frames, ctypes.byref(h))
        if status:
            raise OracleError(status)
        self._h = h

    def read(self, layer: int, heads: int, head_dim: int = 64):
        keys = np.empty((self.frames, heads, head_dim), dtype=np.int8)
        values = np.empty_like(keys)
        ks = np.empty((self.frames, heads), dtype=np.float32)
        vs = np.empty_like(ks)
        lib().nbo_cross_memory_read(self._h, layer, _ptr(keys), _ptr(ks), _ptr(values), _ptr(vs))
        return keys, ks, values, vs

    def __del__(self):
        if getattr(self, "_h", None):
            lib().nbo_cross_memory_free(self._h)
            self._h = None


def text_vocab(model: Model) -> int:
    return int(lib().nbo_model_text_vocab(model._h))
