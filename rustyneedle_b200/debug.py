"""Kernel-level test hooks (include/needle_b200_debug.h): single kernels of the
library run on their own so the tests can compare them with the CPU restatement."""

from __future__ import annotations

import ctypes

import numpy as np

from ._native import Model, Session, _check, _ptr, lib

OP_EXPF, OP_SIGMOID, OP_FAST_EXP, OP_SILU, OP_SINKHORN_RCP = 0, 1, 2, 3, 4
MATRIX_QKVG, MATRIX_OUT, MATRIX_LOGITS = 0, 1, 2

_declared = False


def _declare() -> None:
    global _declared
    if _declared:
        return
    L = lib()
    P, SZ, U32, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_int
    for name, args in {
        "nb_debug_math": [P, I, P, P, SZ],
        "nb_debug_project": [P, I, U32, P, SZ, P],
        "nb_debug_hidden": [P, P],
        "nb_debug_hadamard": [P, U32, P, SZ, P],
        "nb_debug_kv": [P, U32, P, P, P, P],
        "nb_debug_time_attention": [P, U32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double)],
        "nb_debug_cross_memory": [P, ctypes.c_int, P, P, P, P],
        "nb_debug_step_kernels": [P, ctypes.POINTER(ctypes.c_uint32)],
        "nb_debug_product": [I, U32, P, P, P, U32, U32, P, U32, P, U32, ctypes.POINTER(ctypes.c_float)],
        "nb_debug_read_bandwidth": [I, SZ, U32, U32, ctypes.POINTER(ctypes.c_float)],
        "nb_debug_expire_waits": [P, U32],
    }.items():
        fn = getattr(L, name)
        fn.restype = I
        fn.argtypes = args
    _declared = True


def math(model: Model, op: int, x: np.ndarray) -> np.ndarray:
    _declare()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _check(lib().nb_debug_math(model._h, op, _ptr(x), _ptr(out), x.size))
    return out


def project(model: Model, which: int, layer: int, x: np.ndarray, rows: int) -> np.ndarray:
    _declare()
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    out = np.empty((x.shape[0], rows), dtype=np.float32)
    _check(lib().nb_debug_project(model._h, which, layer, _ptr(x), x.shape[0], _ptr(out)))
    return out


def hadamard(model: Model, layer: int, x: np.ndarray) -> np.ndarray:
    _declare()
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    out = np.empty_like(x)
    _check(lib().nb_debug_hadamard(model._h, layer, _ptr(x), x.shape[0], _ptr(out)))
    return out


def hidden(session: Session) -> np.ndarray:
    _declare()
    out = np.empty(session.model.config.d_model, dtype=np.float32)
    _check(lib().nb_debug_hidden(session._h, _ptr(out)))
    return out


def kv(session: Session, layer: int):
    _declare()
    c = session.model.config
    n = len(session)
    keys = np.zeros((n, c.num_kv_heads, c.head_dim), dtype=np.int8)
    values = np.zeros_like(keys)
    ks = np.zeros((c.num_kv_heads, n), dtype=np.float32)
    vs = np.zeros_like(ks)
    _check(lib().nb_debug_kv(session._h, layer, _ptr(keys), _ptr(ks), _ptr(values), _ptr(vs)))
    return keys, ks, values, vs


def cross_memory(memory, layer: int, heads: int, head_dim: int = 64):
    """A cross memory's keys, key scales, values and value scales of one layer."""
    _declare()
    keys = np.empty((memory.frames, heads, head_dim), dtype=np.int8)
    values = np.empty_like(keys)
    ks = np.empty((memory.frames, heads), dtype=np.float32)
    vs = np.empty_like(ks)
    _check(lib().nb_debug_cross_memory(memory._h, layer, keys.ctypes.data, ks.ctypes.data, values.ctypes.data, vs.ctypes.data))
    return keys, ks, values, vs


def time_attention(batch, reps: int = 5):
    """Mean device ms of one attention launch over the batch's current
    positions, and the KV bytes that launch reads."""
    _declare()
    ms, nbytes = ctypes.c_float(), ctypes.c_double()
    _check(lib().nb_debug_time_attention(batch._h, reps, ctypes.byref(ms), ctypes.byref(nbytes)))
    return float(ms.value), float(nbytes.value)


def step_kernels(batch) -> int:
    """Kernels in the batch's step graph (0 before its first step)."""
    _declare()
    n = ctypes.c_uint32()
    _check(lib().nb_debug_step_kernels(batch._h, ctypes.byref(n)))
    return int(n.value)


def product(bits: int, packed: np.ndarray, levels: np.ndarray, norms: np.ndarray, rows: int, cols: int, x: np.ndarray,
            reps: int = 0, device: int = 0):
    """The product microbenchmark: outputs (count × rows) and, with reps > 0,
    the mean device milliseconds of the product kernel alone."""
    _declare()
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    lv = np.ascontiguousarray(levels, dtype=np.float32)
    nm = np.ascontiguousarray(norms, dtype=np.uint16)
    xv = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    out = np.empty((xv.shape[0], rows), dtype=np.float32)
    ms = ctypes.c_float()
    _check(lib().nb_debug_product(device, bits, _ptr(p), _ptr(lv), _ptr(nm), rows, cols, _ptr(xv), xv.shape[0], _ptr(out), reps,
                                  ctypes.byref(ms)))
    return out, float(ms.value)


def read_bandwidth(nbytes: int, passes: int = 1, reps: int = 20, device: int = 0) -> float:
    """GB/s of a plain streaming read of an `nbytes` device buffer, read
    `passes` times per launch (the mean over `reps` launches): the L2 read
    peak below the L2 size, HBM above it."""
    _declare()
    ms = ctypes.c_float()
    _check(lib().nb_debug_read_bandwidth(device, nbytes, passes, reps, ctypes.byref(ms)))
    return nbytes / (ms.value / 1000.0) / 1e9


def expire_waits(model: Model, count: int = 1) -> None:
    """The next `count` routing CTAs give up a bounded wait (nb_debug_expire_waits)."""
    _declare()
    _check(lib().nb_debug_expire_waits(model._h, count))
