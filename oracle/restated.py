"""A second CPU restatement of the token loop's composite arithmetic, in numpy.

Test infrastructure only: nothing in the product imports it. It is written
from the Rust source of the reference (the aarch64 integer branches, which
the C++ restatement in needle_oracle.cpp calls INT mode) and is used by
tests/test_oracle_restated.py to cross-check that restatement on the paths
no reference test vector pins: the codebook products with their per-group
combine, one head's attention with its 12-bit value weights, the Sinkhorn
mixing and the grammar step's allowed statistics. Every function names the
reference lines it follows. Arithmetic is f32 throughout, one rounding per
Rust operation, in the Rust order.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import math

import numpy as np

F32 = np.float32
GROUP = 128
COEFFICIENT_LEVELS = F32(2047.0)  # crates/kernels/src/attention.rs:3
LOG2_E = F32(math.log2(math.e))  # std::f32::consts::LOG2_E
LN_2 = F32(math.log(2.0))  # std::f32::consts::LN_2
MIN_POSITIVE = F32(np.finfo(np.float32).tiny)


# ------------------------------------------------------------------ helpers
def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """a·b + c with one rounding to f32 (NEON vfmaq_f32), elementwise.

    a·b of two f32 values is exact in f64; the f64 sum s and its exact error
    e (Knuth's two-sum) give the exact a·b + c = s + e. Rounding s to f32
    is the correct rounding of s + e except when s is exactly halfway
    between two f32 neighbours and e != 0; then the neighbour on e's side is
    the answer."""
    p = np.asarray(a, dtype=np.float64) * np.asarray(b, dtype=np.float64)
    t = np.asarray(c, dtype=np.float64)
    s = p + t
    bb = s - p
    e = (p - (s - bb)) + (t - bb)
    r = s.astype(np.float32)
    toward = np.where(s > r.astype(np.float64), np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    other = np.nextafter(r, toward)
    midpoint = (r.astype(np.float64) != s) & ((r.astype(np.float64) + other.astype(np.float64)) / 2.0 == s)
    fix = midpoint & (e != 0.0) & (np.sign(other.astype(np.float64) - s) == np.sign(e))
    return np.where(fix, other, r).astype(np.float32)


def round_half_away(x: np.ndarray) -> np.ndarray:
    """f32::round / vrndaq_f32 / vcvtaq_s32_f32: nearest, ties away from zero
    (computed in f64, where |x| + 0.5 is exact for these magnitudes)."""
    x64 = np.asarray(x, dtype=np.float64)
    return np.sign(x64) * np.floor(np.abs(x64) + 0.5)


def half_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def walsh(values: np.ndarray) -> np.ndarray:
    """walsh::transform_in_place (crates/kernels/src/walsh.rs:45-80; the
    128-wide NEON form at :17-37 forms the same sums): the quad step, then
    butterflies of doubling span, then times 1/sqrt(length)."""
    v = np.array(values, dtype=np.float32)
    n = v.size
    a, b, c, d = v[0::4].copy(), v[1::4].copy(), v[2::4].copy(), v[3::4].copy()
    low_sum, low_difference = a + b, a - b
    high_sum, high_difference = c + d, c - d
    v[0::4] = low_sum + high_sum
    v[1::4] = low_difference + high_difference
    v[2::4] = low_sum - high_sum
    v[3::4] = low_difference - high_difference
    span = 4
    while span < n:
        blocks = v.reshape(-1, 2 * span)
        low, high = blocks[:, :span].copy(), blocks[:, span:].copy()
        blocks[:, :span] = low + high
        blocks[:, span:] = low - high
        v = blocks.reshape(-1)
        span *= 2
    scale = F32(1.0) / np.sqrt(F32(n))
    return (v * scale).astype(np.float32)


def peak_magnitude(values: np.ndarray) -> np.float32:
    """ops::peak_magnitude (crates/kernels/src/ops.rs:32-42): max |x| from 0.0."""
    v = np.abs(np.asarray(values, dtype=np.float32))
    return F32(max(F32(0.0), v.max())) if v.size else F32(0.0)


# ---------------------------------------------------------- codebook products
def integer_levels(levels: np.ndarray, count: int):
    """IntegerLevels::new (crates/kernels/src/neon.rs:110-121): the levels as
    int8 multiples of peak/127, rounded half away from zero."""
    lv = np.zeros(16, dtype=np.float32)
    lv[:count] = np.asarray(levels, dtype=np.float32)[:count]
    peak = peak_magnitude(lv[:count])
    scale = peak / F32(127.0) if peak > 0 else F32(1.0)
    table = np.zeros(16, dtype=np.int64)
    table[:count] = round_half_away(lv[:count] / scale).astype(np.int64)
    return table, F32(scale)


def quantise_groups(rotated: np.ndarray, group: int = GROUP):
    """The activation of one row (NaturalInput::new, panel.rs:48-66, and
    PlaneInput::four_bit, neon.rs:73-87): per group scale = peak/127 (1 when
    the group is zero) and codes = x / scale rounded half to even, clamped to
    [-127, 127] (quantise_sixteen, neon.rs:23-34)."""
    x = np.asarray(rotated, dtype=np.float32).reshape(-1, group)
    peaks = np.abs(x).max(axis=1)
    scales = np.where(peaks > 0, peaks / F32(127.0), F32(1.0)).astype(np.float32)
    q = x / scales[:, None]
    codes = np.clip(np.rint(q), -127, 127).astype(np.int64)  # rint: ties to even
    return codes, scales


def unpack_codes(packed: np.ndarray, bits: int, rows: int, cols: int) -> np.ndarray:
    """LookupTable::value (crates/kernels/src/matrix.rs:621-630): element i of
    a row at bit offset i·bits, least significant bits first."""
    p = np.asarray(packed, dtype=np.uint8).reshape(rows, cols * bits // 8)
    per = 8 // bits
    mask = (1 << bits) - 1
    out = np.zeros((rows, cols), dtype=np.int64)
    for k in range(per):
        out[:, k::per] = (p >> (k * bits)) & mask
    return out


def product_int(bits: int, packed: np.ndarray, levels: np.ndarray, norms: np.ndarray, rows: int, cols: int,
                x: np.ndarray) -> np.ndarray:
    """QuantisedMatrix::prepare + multiply_vector on the integer kernels
    (crates/kernels/src/matrix.rs:123-165, :342-363), for 2- and 4-bit
    codebooks with 128-column groups.

    The input is rotated per group (walsh) and quantised per group; each
    (row, group) sum Σ level_code · activation_code is exact in integers.
    The combine differs by width. 2-bit rows run as panels (panel.rs:168-190):
    total = fma(sum, (norm · level_scale) · act_scale, total). 4-bit rows run
    row_dot_four_bit (neon.rs:196-216): total += ((sum · norm) · level_scale)
    · act_scale. Both start from +0.0 and go in group order."""
    groups = cols // GROUP
    rotated = np.concatenate([walsh(g) for g in np.asarray(x, dtype=np.float32).reshape(groups, GROUP)])
    act, act_scales = quantise_groups(rotated)
    table, level_scale = integer_levels(levels, 1 << bits)
    codes = table[unpack_codes(packed, bits, rows, cols)]  # [rows][cols] int8 levels
    sums = np.einsum("rgk,gk->rg", codes.reshape(rows, groups, GROUP), act)  # exact int64
    norm = half_to_f32(norms).reshape(rows, groups)
    total = np.zeros(rows, dtype=np.float32)
    for g in range(groups):
        s = sums[:, g].astype(np.float32)
        if bits == 2:
            scaled = (norm[:, g] * level_scale).astype(np.float32) * act_scales[g]
            total = fma_f32(s, scaled.astype(np.float32), total)
        else:
            term = ((s * norm[:, g]).astype(np.float32) * level_scale).astype(np.float32) * act_scales[g]
            total = (total + term.astype(np.float32)).astype(np.float32)
    return total


# ------------------------------------------------------------------ attention
def fast_exp(values: np.ndarray) -> np.ndarray:
    """ops::fast_exp (crates/kernels/src/ops.rs:83-90), which exp_neon
    (neon.rs:262-274) evaluates lane by lane with the same operations."""
    v = np.clip(np.asarray(values, dtype=np.float32), F32(-87.0), F32(87.0))
    scaled = (v * LOG2_E).astype(np.float32)
    whole = round_half_away(scaled).astype(np.float32)
    fraction = (scaled - whole).astype(np.float32)
    p = np.full_like(fraction, F32(0.001_333_355_8))
    for coefficient in (F32(0.009_618_129), F32(0.055_504_11), F32(0.240_226_5), LN_2, F32(1.0)):
        p = ((p * fraction).astype(np.float32) + coefficient).astype(np.float32)
    return (p * np.ldexp(np.float32(1.0), whole.astype(np.int32)).astype(np.float32)).astype(np.float32)


def attend_head_int(query: np.ndarray, query_scale: float, keys: np.ndarray, key_scales: np.ndarray,
                    values: np.ndarray, value_scales: np.ndarray) -> np.ndarray:
    """attend_head on the integer kernels (crates/kernels/src/attention.rs:53-77).

    Scores q·k exact; coefficients (score · key_scale) · query_scale; the
    peak; e = fast_exp(c - peak) with the total formed as NEON does
    (softmax_inner, neon.rs:277-307): four lanes of every fourth position
    over the whole quads, summed (l0 + l1) + (l2 + l3), then the tail
    positions one by one; weights e · value_scale. The weights become
    integers w / (peak|w| / 2047) rounded half away (split_coefficients,
    neon.rs:348-366), whose sums with the value codes are exact
    (accumulate_panel_chunks, neon.rs:368-393); the output is that sum
    times the scale, times 1 / total."""
    q = np.asarray(query, dtype=np.int64)
    k = np.asarray(keys, dtype=np.int64)
    v = np.asarray(values, dtype=np.int64)
    ks = np.asarray(key_scales, dtype=np.float32)
    vs = np.asarray(value_scales, dtype=np.float32)
    count = k.shape[0]
    scores = (k @ q).astype(np.float32)
    coefficients = ((scores * ks).astype(np.float32) * F32(query_scale)).astype(np.float32)
    peak = coefficients.max()
    e = fast_exp((coefficients - peak).astype(np.float32))
    quads = count - count % 4
    lanes = [F32(0.0)] * 4
    for i in range(quads):
        lanes[i % 4] = F32(lanes[i % 4] + e[i])
    total = F32(F32(lanes[0] + lanes[1]) + F32(lanes[2] + lanes[3]))
    for i in range(quads, count):
        total = F32(total + e[i])
    weights = (e * vs).astype(np.float32)
    width = v.shape[1]
    peak_w = peak_magnitude(weights)
    if peak_w <= 0:
        out = np.zeros(width, dtype=np.float32)
    else:
        scale = F32(peak_w / COEFFICIENT_LEVELS)
        integer = round_half_away((weights / scale).astype(np.float32)).astype(np.int64)
        sums = integer @ v  # exact
        out = (sums.astype(np.float32) * scale).astype(np.float32)
    inverse = F32(F32(1.0) / total)
    return (out * inverse).astype(np.float32)


# ------------------------------------------------------------------ sinkhorn
_libm = ctypes.CDLL(ctypes.util.find_library("m"))
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]


def expf(x: float) -> np.float32:
    """f32::exp, which Rust takes from the platform's libm (here glibc)."""
    return F32(_libm.expf(float(x)))


def sinkhorn(logits: np.ndarray, size: int, iterations: int = 20) -> np.ndarray:
    """ops::sinkhorn_in_place (crates/kernels/src/ops.rs:198-217): per row
    exp(x - peak); then per iteration every row and then every column times
    1 / max(total, MIN_POSITIVE), the totals ordered f32 sums from -0.0
    (Iterator::sum)."""
    m = np.array(logits, dtype=np.float32).reshape(size, size)
    for r in range(size):
        peak = m[r].max()
        for c in range(size):
            m[r, c] = expf(F32(m[r, c] - peak))
    for _ in range(iterations):
        for r in range(size):
            total = F32(-0.0)
            for c in range(size):
                total = F32(total + m[r, c])
            inverse = F32(F32(1.0) / max(total, MIN_POSITIVE))
            m[r] = (m[r] * inverse).astype(np.float32)
        for c in range(size):
            total = F32(-0.0)
            for r in range(size):
                total = F32(total + m[r, c])
            inverse = F32(F32(1.0) / max(total, MIN_POSITIVE))
            m[:, c] = (m[:, c] * inverse).astype(np.float32)
    return m.reshape(-1)


# ------------------------------------------------------------ grammar step
def allowed_statistics(logits: np.ndarray, token: int, allowed: np.ndarray):
    """allowed_statistics (crates/generate/src/generator.rs:178-194): peaks
    over all ids and over the allowed ones; two totals of fast_exp from +0.0
    in id order (the allowed one times 1.0 or 0.0); the chosen token's
    probability and the allowed mass."""
    x = np.asarray(logits, dtype=np.float32)
    ok = np.asarray(allowed, dtype=bool)
    peak_all = x.max()
    peak_allowed = np.where(ok, x, F32(-np.inf)).max()
    e_all = fast_exp((x - peak_all).astype(np.float32))
    e_allowed = (fast_exp((x - peak_allowed).astype(np.float32)) * ok.astype(np.float32)).astype(np.float32)
    total_all, total_allowed = F32(0.0), F32(0.0)
    for i in range(x.size):
        total_all = F32(total_all + e_all[i])
        total_allowed = F32(total_allowed + e_allowed[i])
    probability = F32(fast_exp(np.array([x[token] - peak_allowed], dtype=np.float32))[0] / total_allowed)
    mass = F32(F32(total_allowed * fast_exp(np.array([peak_allowed - peak_all], dtype=np.float32))[0]) / total_all)
    return probability, mass
