"""A second CPU restatement of the token loop's composite arithmetic, in numpy.

Test infrastructure only: nothing in the product imports it. It is written
from the Rust source of the reference (the aarch64 integer branches, which
the C++ restatement in needle_oracle.cpp calls INT mode) and is used by
tests/test_oracle_restated.py to cross-check that restatement on the paths
no reference test vector pins: the codebook products with their per-group
combine, one head's attention with its 12-bit value weights, the Sinkhorn
mixing, the grammar step's allowed statistics, a layer's Hadamard block
(condition softmax, modulation, three Kronecker factor pairs) and its lane
routing (the phi products, the gates with the own-lane offsets), and from
them a whole token: Session::push (every layer's lane stream) and
Session::logits, with the Whistle cross attention (the cross memory and
CrossState::apply) when a memory is given. It reads the archive with its
own reader. Every function
names the
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


# ------------------------------------------------------------ archive reader
class Archive:
    """The tensors of a .cact file, read with numpy (crates/cact/src/geometry.rs:41-90,
    record.rs:38-50): 48 u32 header fields (the tensor count second, the
    codebook length third) and the f32 rope theta, 196 bytes; the codebook
    floats; one 44-byte record per tensor (kind u8, rank u8, u16, four u32
    dims, u64 offset, u64 byte length, u32 group, u32 bits); tensor bytes at
    their offsets. The tensors come in the order of crates/cact/src/layout.rs:
    the embedding, then per layer norm_in, q/k/v, [3 conv taps], q_norm,
    k_norm, gate_proj, out_proj, post_norm, attn_gate, pre_hada and 13
    Hadamard tensors (:199-210), then the 9 lane tensors and the two
    Hadamard permutations (:186-189)."""

    HEADER_BYTES, RECORD_BYTES = 196, 44
    SINGLE, CODEBOOK = 2, 3

    def __init__(self, path: str):
        import struct

        with open(path, "rb") as f:
            self.data = f.read()
        fields = struct.unpack_from("<48I", self.data, 0)
        self.count, codebook_len = fields[1], fields[2]
        self.layers, self.d_model, self.lanes, self.conv_taps = fields[10], fields[7], fields[15], fields[19]
        # engram geometry (crates/cact/src/geometry.rs:66-82): slots, sub_dim, tables,
        # conv taps, dilation, seed heads, the orders, the site layers
        self.engram = dict(slots=fields[20], sub_dim=fields[21], tables=fields[22], conv_taps=fields[23], dilation=fields[24],
                           seed_heads=fields[25], orders=list(fields[27:27 + fields[26]]), sites=list(fields[32:32 + fields[31]]))
        self.codebook = np.frombuffer(self.data, "<f4", codebook_len, self.HEADER_BYTES).astype(np.float32)
        at = self.HEADER_BYTES + codebook_len * 4
        self.records = [struct.unpack_from("<BBH4IQQII", self.data, at + self.RECORD_BYTES * i) for i in range(self.count)]

    def floats(self, index: int) -> np.ndarray:
        kind, rank, _, *rest = self.records[index]
        offset, nbytes = rest[4], rest[5]
        assert kind == self.SINGLE, (index, kind)
        return np.frombuffer(self.data, "<f4", nbytes // 4, offset).astype(np.float32)

    def codebook_matrix(self, index: int):
        """(bits, packed [rows × row bytes], the 2^bits levels, fp16 norms, rows, columns)."""
        kind, rank, _, rows, cols, _, _, offset, nbytes, group, bits = self.records[index]
        assert kind == self.CODEBOOK and group == GROUP, (index, kind, group)
        packed_len = rows * cols * bits // 8
        packed = np.frombuffer(self.data, np.uint8, packed_len, offset)
        norms = np.frombuffer(self.data, "<u2", (nbytes - packed_len) // 2, offset + packed_len)
        first = {2: 0, 3: 4, 4: 12}[bits]  # two-, three-, four-bit levels (crates/kernels/src/codebook.rs:13-19)
        return bits, packed, self.codebook[first:first + (1 << bits)], norms, rows, cols

    def layer_base(self, layer: int) -> int:
        return 1 + layer * (21 + (3 if self.conv_taps else 0) + 3)

    def hadamard(self, layer: int):
        base = self.layer_base(layer) + (14 if self.conv_taps else 11)
        names = ("d1", "d2", "b2", "d3", "d4", "w1a", "w1b", "w2a", "w2b", "w3a", "w3b", "cond_v", "cond_u")
        t = {name: self.floats(base + i) for i, name in enumerate(names)}
        lanes = self.layer_base(self.layers)
        t["perms"] = [self.floats(lanes + 9).astype(np.int64), self.floats(lanes + 10).astype(np.int64)]
        return t

    def engram_tensors(self, site: int) -> dict:
        """Site `site`'s tables, key_proj, value_proj and taps (layout.rs:231-234),
        after the lane tensors and the two Hadamard permutations."""
        base = self.layer_base(self.layers) + 11 + 4 * site
        return dict(tables=self.codebook_matrix(base), key=self.codebook_matrix(base + 1), value=self.codebook_matrix(base + 2),
                    taps=self.floats(base + 3))

    def final_norm_index(self) -> int:
        return self.layer_base(self.layers) + 11 + 4 * len(self.engram["sites"])

    def head_tensors(self) -> list:
        """The probe heads (crates/cact/src/layout.rs:236-254): a half-precision
        manifest of head codes after the final norm, then per head probes,
        gain, query, row_bias, proj and bias (and a calibration for code 3)."""
        at = self.final_norm_index() + 1
        if at >= self.count or self.records[at][0] != 1:
            return []
        _, _, _, n, _, _, _, offset, nbytes, _, _ = self.records[at]
        codes = np.frombuffer(self.data, "<f2", n, offset).astype(np.float32)
        heads, at = [], at + 1
        for code in codes:
            heads.append(dict(code=int(code), probes=self.codebook_matrix(at), gain=self.floats(at + 1), query=self.codebook_matrix(at + 2),
                              row_bias=self.floats(at + 3), proj=self.codebook_matrix(at + 4), bias=self.floats(at + 5)))
            at += 6 + (1 if int(code) == 3 else 0)
        return heads

    def audio_index(self) -> int:
        """The audio manifest's record: after the final norm and the probe heads."""
        at = self.final_norm_index() + 1
        if at < self.count and self.records[at][0] == 1:
            codes = np.frombuffer(self.data, "<f2", self.records[at][3], self.records[at][7]).astype(np.float32)
            at += 1 + sum(6 + (1 if int(c) == 3 else 0) for c in codes)
        return at

    def lane_tensors(self):
        base = self.layer_base(self.layers)
        names = ("a_pre", "a_post", "a_res", "b_pre", "b_post", "b_res")
        t = {name: self.floats(base + i) for i, name in enumerate(names)}
        for i, name in enumerate(("phi_pre", "phi_post", "phi_res")):
            t[name] = self.codebook_matrix(base + 6 + i)
        return t


# --------------------------------------------------------- Hadamard block
def kronecker32(values: np.ndarray, left: np.ndarray, right: np.ndarray) -> np.ndarray:
    """kronecker_apply_fixed::<32> (crates/kernels/src/ops.rs:143-163), the
    form both architectures run when the left factor is not 32 wide: mixed
    row i = Σ_j x[i][j] · right[j] in j order, then output row k =
    Σ_i left[i][k] · mixed[i] in i order; every sum from +0.0, a multiply and
    an add per term."""
    R = 32
    left_size = int(round(math.sqrt(left.size)))
    x = np.asarray(values, dtype=np.float32).reshape(left_size, R)
    rt = np.asarray(right, dtype=np.float32).reshape(R, R)
    lf = np.asarray(left, dtype=np.float32).reshape(left_size, left_size)
    mixed = np.zeros((left_size, R), dtype=np.float32)
    for j in range(R):
        mixed = (mixed + (x[:, j:j + 1] * rt[j][None, :]).astype(np.float32)).astype(np.float32)
    out = np.zeros((left_size, R), dtype=np.float32)
    for i in range(left_size):
        out = (out + (lf[i][:, None] * mixed[i][None, :]).astype(np.float32)).astype(np.float32)
    return out.reshape(-1)


def silu(values: np.ndarray) -> np.ndarray:
    """ops::silu (crates/kernels/src/ops.rs:74-76): x / (1 + fast_exp(-x))."""
    v = np.asarray(values, dtype=np.float32)
    return (v / (F32(1.0) + fast_exp(-v)).astype(np.float32)).astype(np.float32)


def hadamard_apply(t: dict, x: np.ndarray) -> np.ndarray:
    """HadamardWeights::apply (crates/model/src/hadamard.rs:55-99).

    Condition weights: with rank 8, four chains (dimension d feeds chain
    d mod 4, in order) of products with cond_v, then the chains added in
    order; softmax_in_place (ops.rs:92-101) of them; the modulation
    1 + Σ_rank weight · cond_u. The input padded to the factor size, times
    d1, through factor pair 1, gathered by the first permutation,
    silu(d2 · modulation · gathered + b2), factor pair 2, the second
    permutation, times d3, factor pair 3, times d4, the first width kept."""
    x = np.asarray(x, dtype=np.float32)
    width, size = x.size, t["d1"].size
    rank = t["cond_u"].size // size
    cond_v = t["cond_v"].reshape(width, rank)
    weights = np.zeros(rank, dtype=np.float32)
    if rank == 8:
        chains = np.zeros((4, rank), dtype=np.float32)
        for d in range(width):
            chains[d % 4] = (chains[d % 4] + (x[d] * cond_v[d]).astype(np.float32)).astype(np.float32)
        for c in range(4):
            weights = (weights + chains[c]).astype(np.float32)
    else:
        for d in range(width):
            weights = (weights + (x[d] * cond_v[d]).astype(np.float32)).astype(np.float32)
    peak = weights.max()
    e = fast_exp((weights - peak).astype(np.float32))
    total = F32(0.0)
    for v in e:
        total = F32(total + v)
    weights = (e * F32(F32(1.0) / total)).astype(np.float32)
    cond_u = t["cond_u"].reshape(rank, size)
    modulation = np.ones(size, dtype=np.float32)
    for r in range(rank):
        modulation = (modulation + (weights[r] * cond_u[r]).astype(np.float32)).astype(np.float32)
    padded = np.zeros(size, dtype=np.float32)
    padded[:width] = x
    first = kronecker32((padded * t["d1"]).astype(np.float32), t["w1a"], t["w1b"])
    gathered = first[t["perms"][0]]
    inner = (((t["d2"] * modulation).astype(np.float32) * gathered).astype(np.float32) + t["b2"]).astype(np.float32)
    second = kronecker32(silu(inner), t["w2a"], t["w2b"])
    third = kronecker32((second[t["perms"][1]] * t["d3"]).astype(np.float32), t["w3a"], t["w3b"])
    return (third * t["d4"]).astype(np.float32)[:width]


# ------------------------------------------------------------------ routing
def sum_of_squares(values: np.ndarray) -> np.float32:
    """ops::sum_of_squares (crates/kernels/src/ops.rs:7-17): eight lanes of
    every eighth square, the lanes summed in order from -0.0, plus the tail."""
    v = np.asarray(values, dtype=np.float32)
    whole = v.size - v.size % 8
    lanes = np.zeros(8, dtype=np.float32)
    for i in range(0, whole, 8):
        lanes = (lanes + (v[i:i + 8] * v[i:i + 8]).astype(np.float32)).astype(np.float32)
    total = F32(-0.0)
    for lane in lanes:
        total = F32(total + lane)
    tail = F32(-0.0)
    for value in v[whole:]:
        tail = F32(tail + F32(value * value))
    return F32(total + tail)


def unit_rms(values: np.ndarray) -> np.ndarray:
    """ops::unit_rms (crates/kernels/src/ops.rs:60-66), epsilon 1e-6."""
    v = np.asarray(values, dtype=np.float32)
    mean_square = F32(sum_of_squares(v) / F32(v.size))
    inverse = F32(F32(1.0) / np.sqrt(F32(mean_square + F32(1e-6))))
    return (v * inverse).astype(np.float32)


def fake_quantise_int8(values: np.ndarray) -> np.ndarray:
    """ops::fake_quantise_int8 (crates/kernels/src/ops.rs:120-125)."""
    v = np.asarray(values, dtype=np.float32)
    peak = peak_magnitude(v)
    scale = F32(peak / F32(127.0)) if peak > 0 else F32(1.0)
    return (np.clip(np.rint((v / scale).astype(np.float32)), -128, 127).astype(np.float32) * scale).astype(np.float32)


def sigmoid(value) -> np.float32:
    """ops::sigmoid (crates/kernels/src/ops.rs:69-71) with libm's expf."""
    return F32(F32(1.0) / F32(F32(1.0) + expf(-F32(value))))


def product_rows(matrix, first_row: int, rows: int, x: np.ndarray) -> np.ndarray:
    """Rows first_row.. of a codebook matrix times x (multiply_fused,
    crates/kernels/src/matrix.rs:167-193, row by row as product_int)."""
    bits, packed, levels, norms, all_rows, cols = matrix
    row_bytes = cols * bits // 8
    groups = cols // GROUP
    return product_int(bits, packed[first_row * row_bytes:(first_row + rows) * row_bytes], levels,
                       norms[first_row * groups:(first_row + rows) * groups], rows, cols, x)


def route(lt: dict, lanes: int, layer: int, slot: int, stream: np.ndarray):
    """LaneWeights::route (crates/model/src/lanes.rs:45-80): the stream
    unit-normalised and fake-quantised; the phi products of this layer's
    rows; the pre gates sigmoid(a_pre · pre + b_pre + offset) (own lane
    8 - 4, others -4), the block input Σ_lane gate · lane from +0.0; the post
    gates 2 · sigmoid(a_post · post + b_post + offset) (own lane 0, others
    -4); the residual mixing a_res · r + b_res through the Sinkhorn."""
    s = np.asarray(stream, dtype=np.float32)
    width = s.size // lanes
    normalised = fake_quantise_int8(unit_rms(s))
    pre = product_rows(lt["phi_pre"], layer * lanes, lanes, normalised)
    post = product_rows(lt["phi_post"], layer * lanes, lanes, normalised)
    residual = product_rows(lt["phi_res"], layer * lanes * lanes, lanes * lanes, normalised)
    own = slot % lanes
    block_input = np.zeros(width, dtype=np.float32)
    post_gates = np.zeros(lanes, dtype=np.float32)
    for lane in range(lanes):
        pre_offset = F32(8.0 + -4.0) if lane == own else F32(-4.0)
        gate = sigmoid(F32(F32(F32(lt["a_pre"][layer] * pre[lane]) + lt["b_pre"][layer * lanes + lane]) + pre_offset))
        block_input = (block_input + (gate * s[lane * width:(lane + 1) * width]).astype(np.float32)).astype(np.float32)
        post_offset = F32(0.0) if lane == own else F32(-4.0)
        post_gates[lane] = F32(2.0) * sigmoid(F32(F32(F32(lt["a_post"][layer] * post[lane]) + lt["b_post"][layer * lanes + lane]) + post_offset))
    base = layer * lanes * lanes
    mixed = ((lt["a_res"][layer] * residual).astype(np.float32) + lt["b_res"][base:base + lanes * lanes]).astype(np.float32)
    return block_input, post_gates, sinkhorn(mixed, lanes)


# ------------------------------------------------------------ a whole token
_libm.sinf.restype = _libm.cosf.restype = _libm.powf.restype = ctypes.c_float
_libm.sinf.argtypes = _libm.cosf.argtypes = [ctypes.c_float]
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]


def dequantise_row(matrix, row: int) -> np.ndarray:
    """QuantisedMatrix::dequantise_row (crates/kernels/src/matrix.rs:140-152):
    level × norm per element, then the Walsh transform per group."""
    bits, packed, levels, norms, rows, cols = matrix
    row_bytes = cols * bits // 8
    codes = unpack_codes(packed[row * row_bytes:(row + 1) * row_bytes], bits, 1, cols)[0]
    norm = half_to_f32(norms[row * (cols // GROUP):(row + 1) * (cols // GROUP)])
    lv = np.asarray(levels, dtype=np.float32)
    return np.concatenate([walsh((lv[codes[g * GROUP:(g + 1) * GROUP]] * norm[g]).astype(np.float32)) for g in range(cols // GROUP)])


def engram_indices(cfg: dict, tokens: list, position: int) -> list:
    """table_indices (crates/model/src/engram.rs:30-45): per order and head a
    32-bit hash seeded by 0x9E3779B9 · (order_index · stride + head + 1), each
    of the last `order` tokens (0 before the start) xored in and multiplied by
    0x01000193, then xored with itself shifted right 15, modulo the slots."""
    heads_per_order = cfg["tables"] // max(1, len(cfg["orders"]))
    stride = heads_per_order if cfg["seed_heads"] == 0 else cfg["seed_heads"]
    mask = 0xFFFFFFFF
    out = []
    for order_index, order in enumerate(cfg["orders"]):
        for head in range(heads_per_order):
            acc = (0x9E3779B9 * (order_index * stride + head + 1)) & mask
            for back in range(order):
                token = tokens[position - back] if position >= back else 0
                acc = ((acc ^ token) * 0x01000193) & mask
            acc ^= acc >> 15
            out.append(acc % cfg["slots"])
    return out


def lane_mean(stream: np.ndarray, lanes: int) -> np.ndarray:
    """lane_mean (crates/model/src/session.rs:191-199): Σ_lane value / lanes from +0.0."""
    s = np.asarray(stream, dtype=np.float32).reshape(lanes, -1)
    mean = np.zeros(s.shape[1], dtype=np.float32)
    for lane in s:
        mean = (mean + (lane / F32(lanes)).astype(np.float32)).astype(np.float32)
    return mean


def dot_product(a: np.ndarray, b: np.ndarray) -> np.float32:
    """ops::dot_product (crates/kernels/src/ops.rs:19-30): eight lanes of every
    eighth product, the lanes summed in order from -0.0, plus the tail."""
    x, y = np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32)
    whole = x.size - x.size % 8
    lanes = np.zeros(8, dtype=np.float32)
    for i in range(0, whole, 8):
        lanes = (lanes + (x[i:i + 8] * y[i:i + 8]).astype(np.float32)).astype(np.float32)
    total = F32(-0.0)
    for lane in lanes:
        total = F32(total + lane)
    tail = F32(-0.0)
    for p, q in zip(x[whole:], y[whole:]):
        tail = F32(tail + F32(p * q))
    return F32(total + tail)


class ProbeHead:
    """ProbeHead (crates/model/src/heads.rs): the dense probe and query rows,
    the running per-slot softmax pool of the cells (observe, :129-148), the
    pooled readout (:88-117) and its projection (:119-127)."""

    def __init__(self, t: dict, cells: int):
        self.code = t["code"]
        self.probes = np.stack([dequantise_row(t["probes"], r) for r in range(t["probes"][4])])
        self.query = np.stack([dequantise_row(t["query"], r) for r in range(t["query"][4])])
        self.gain, self.row_bias, self.proj, self.bias = t["gain"], t["row_bias"], t["proj"], t["bias"]
        self.slots, self.width = self.probes.shape
        self.per_cell = self.slots // cells
        self.peak = np.full(self.slots, -np.inf, dtype=np.float32)
        self.total = np.zeros(self.slots, dtype=np.float32)
        self.weighted = np.zeros((self.slots, self.width), dtype=np.float32)

    def observe(self, cells: list) -> None:
        root = np.sqrt(F32(self.width))
        for layer, cell in enumerate(cells):
            for probe in range(self.per_cell):
                slot = layer * self.per_cell + probe
                score = F32(dot_product(cell, self.probes[slot]) / root)
                peak = F32(max(self.peak[slot], score))
                rescale = F32(0.0) if self.peak[slot] == -np.inf else expf(F32(self.peak[slot] - peak))
                weight = expf(F32(score - peak))
                self.total[slot] = F32(F32(self.total[slot] * rescale) + weight)
                self.weighted[slot] = ((self.weighted[slot] * rescale).astype(np.float32) + (weight * cell).astype(np.float32)).astype(np.float32)
                self.peak[slot] = peak

    def pooled(self) -> np.ndarray:
        readouts = np.zeros((self.slots, self.width), dtype=np.float32)
        for slot in range(self.slots):
            inverse = F32(F32(1.0) / self.total[slot])
            readouts[slot] = (unit_rms((self.weighted[slot] * inverse).astype(np.float32)) * self.gain[slot]).astype(np.float32)
        root = np.sqrt(F32(self.width))
        out = np.zeros((self.query.shape[0], self.width), dtype=np.float32)
        for q in range(self.query.shape[0]):
            w = np.array([F32(F32(dot_product(readouts[slot], self.query[q]) / root) + self.row_bias[q * self.slots + slot])
                          for slot in range(self.slots)], dtype=np.float32)
            e = fast_exp((w - w.max()).astype(np.float32))
            total = F32(0.0)
            for v in e:
                total = F32(total + v)
            w = (e * F32(F32(1.0) / total)).astype(np.float32)
            for slot in range(self.slots):
                out[q] = (out[q] + (w[slot] * readouts[slot]).astype(np.float32)).astype(np.float32)
        return out.reshape(-1)

    def project(self, pooled: np.ndarray) -> np.ndarray:
        return (product_rows(self.proj, 0, self.proj[4], pooled) + self.bias).astype(np.float32)


def zero_centred_norm(values: np.ndarray, gains: np.ndarray) -> np.ndarray:
    """ops::zero_centred_norm (crates/kernels/src/ops.rs:44-58): (1 + gain) · x · inverse RMS."""
    v = np.asarray(values, dtype=np.float32)
    mean_square = F32(sum_of_squares(v) / F32(v.size))
    inverse = F32(F32(1.0) / np.sqrt(F32(mean_square + F32(1e-6))))
    return (((F32(1.0) + np.asarray(gains, dtype=np.float32)) * v).astype(np.float32) * inverse).astype(np.float32)


def quantise_int8(values: np.ndarray):
    """ops::quantise_int8 (crates/kernels/src/ops.rs:111-118): codes and scale."""
    v = np.asarray(values, dtype=np.float32)
    peak = peak_magnitude(v)
    scale = F32(peak / F32(127.0)) if peak > 0 else F32(1.0)
    return np.clip(np.rint((v / scale).astype(np.float32)), -128, 127).astype(np.int64), scale


class Session:
    """Session::push and Session::logits (crates/model/src/session.rs:78-175)
    of a Needle-3 archive with any of its features (q/k/v convolution taps,
    sliding-window layers, engram sites, probe heads), on the integer
    kernels: the
    embedding row (dequantised and rotated back, times
    sqrt(d)) in every lane; per layer the routing, the attention
    (AttentionWeights::attend, crates/model/src/attention.rs:98-158, with the
    cache's int8 keys and values), the gated residual, the Hadamard block,
    the block delta and the lane combine (lanes.rs:82-104); the lane mean
    through the final norm; the logits through the tied embedding."""

    def __init__(self, archive: Archive):
        import struct

        a = self.archive = archive
        fields = struct.unpack_from("<48I", a.data, 0)
        self.heads, self.kv_heads, self.head_dim = fields[8], fields[9], fields[11]
        self.sliding_window, self.global_layers = fields[16], fields[17] | fields[18] << 32
        theta = F32(struct.unpack_from("<f", a.data, 192)[0])
        half = self.head_dim // 2
        self.frequencies = np.array(
            [F32(F32(1.0) / F32(_libm.powf(float(theta), float(F32(F32(2.0 * i) / F32(self.head_dim)))))) for i in range(half)],
            dtype=np.float32)
        self.lane_weights = a.lane_tensors()
        self.embedding = a.codebook_matrix(0)
        self.final_norm = a.floats(a.final_norm_index())
        self.tokens = []
        self.engram_history = [[] for _ in a.engram["sites"]]
        self.heads_list = [ProbeHead(t, a.layers + 1) for t in a.head_tensors()]
        self.caches = [dict(keys=[], key_scales=[[] for _ in range(self.kv_heads)], values=[],
                            value_scales=[[] for _ in range(self.kv_heads)]) for _ in range(a.layers)]
        self.position = 0
        self.hidden = None

    def _embedding_row(self, token: int) -> np.ndarray:
        return dequantise_row(self.embedding, token)

    def _engram(self, site: int, position: int) -> tuple:
        """EngramSiteState::contribute (crates/model/src/engram.rs:67-100): the
        tables' rows at the hashed indices (zeros while the position is shorter
        than the order), fake-quantised, the key and raw value products, then the
        value as the dilated causal convolution of the raw values."""
        cfg, t = self.archive.engram, self.archive.engram_tensors(site)
        heads_per_order = cfg["tables"] // max(1, len(cfg["orders"]))
        gathered = []
        for table, index in enumerate(engram_indices(cfg, self.tokens, position)):
            order = cfg["orders"][table // heads_per_order]
            if position + 1 >= order:
                gathered.append(dequantise_row(t["tables"], table * cfg["slots"] + index))
            else:
                gathered.append(np.zeros(cfg["sub_dim"], dtype=np.float32))
        gathered = fake_quantise_int8(np.concatenate(gathered))
        key = product_rows(t["key"], 0, t["key"][4], gathered)
        raw = product_rows(t["value"], 0, t["value"][4], gathered)
        history = self.engram_history[site]
        history.insert(0, raw)
        del history[(cfg["conv_taps"] - 1) * cfg["dilation"] + 1:]
        gains = t["taps"].reshape(cfg["conv_taps"], -1)
        value = np.zeros_like(raw)
        for tap in range(cfg["conv_taps"]):
            back = tap * cfg["dilation"]
            if position >= back:
                value = (value + (gains[tap] * history[back]).astype(np.float32)).astype(np.float32)
        return key, value

    def _rotary(self, head: np.ndarray, position: int) -> np.ndarray:
        """ops::apply_rotary (crates/kernels/src/ops.rs:131-141) with libm sinf/cosf."""
        half = head.size // 2
        out = head.copy()
        for i in range(half):
            angle = F32(F32(position) * self.frequencies[i])
            sin, cos = F32(_libm.sinf(float(angle))), F32(_libm.cosf(float(angle)))
            a, b = head[i], head[half + i]
            out[i] = F32(F32(a * cos) - F32(b * sin))
            out[half + i] = F32(F32(b * cos) + F32(a * sin))
        return out

    def _index(self, layer: int, name: str) -> int:
        """A layer tensor's record (crates/cact/src/layout.rs:199-210): norm_in,
        q/k/v, [three conv tap tensors], q_norm, k_norm, gate_proj, out_proj,
        post_norm, attn_gate, pre_hada."""
        a = self.archive
        taps = 3 if a.conv_taps else 0
        order = {"norm_in": 0, "q": 1, "k": 2, "v": 3, "taps": 4, "q_norm": 4 + taps, "k_norm": 5 + taps, "gate": 6 + taps,
                 "out": 7 + taps, "post_norm": 8 + taps, "attn_gate": 9 + taps, "pre_hada": 10 + taps}
        return a.layer_base(layer) + order[name]

    def _attend(self, layer: int, hidden: np.ndarray) -> np.ndarray:
        a, hd, H, KV = self.archive, self.head_dim, self.heads, self.kv_heads
        idx = lambda name: self._index(layer, name)  # noqa: E731
        quantised = fake_quantise_int8(hidden)
        q = product_rows(a.codebook_matrix(idx("q")), 0, H * hd, quantised)
        k = product_rows(a.codebook_matrix(idx("k")), 0, KV * hd, quantised)
        v = product_rows(a.codebook_matrix(idx("v")), 0, KV * hd, quantised)
        gate = product_rows(a.codebook_matrix(idx("gate")), 0, H * hd, quantised)
        cache = self.caches[layer]
        if a.conv_taps:
            # mix_taps (crates/model/src/attention.rs:83-93, 112-119): the raw
            # projections newest first, then Σ over tap < min(taps, position + 1)
            # of gain[tap] · history[tap] from +0.0
            history = cache.setdefault("history", [])
            history.insert(0, (q, k, v))
            del history[a.conv_taps:]
            mixed = []
            for which in range(3):
                gains = a.floats(idx("taps") + which).reshape(a.conv_taps, -1)
                out = np.zeros_like(history[0][which])
                for tap in range(min(a.conv_taps, self.position + 1)):
                    out = (out + (gains[tap] * history[tap][which]).astype(np.float32)).astype(np.float32)
                mixed.append(out)
            q, k, v = mixed
        q_norm, k_norm = a.floats(idx("q_norm")), a.floats(idx("k_norm"))
        query_codes, query_scales = [], []
        for h in range(H):
            head = self._rotary(zero_centred_norm(q[h * hd:(h + 1) * hd], q_norm), self.position)
            codes, scale = quantise_int8(head)
            query_codes.append(codes)
            query_scales.append(scale)
        keys, values = np.zeros((KV, hd), dtype=np.int64), np.zeros((KV, hd), dtype=np.int64)
        for kv in range(KV):
            head = self._rotary(zero_centred_norm(k[kv * hd:(kv + 1) * hd], k_norm), self.position)
            keys[kv], scale = quantise_int8(head)
            cache["key_scales"][kv].append(scale)
        for kv in range(KV):
            values[kv], scale = quantise_int8(v[kv * hd:(kv + 1) * hd])
            cache["value_scales"][kv].append(scale)
        cache["keys"].append(keys)
        cache["values"].append(values)
        total = self.position + 1
        windowed = self.sliding_window > 0 and not (self.global_layers >> layer & 1)
        first = max(0, total - self.sliding_window) if windowed else 0
        all_keys, all_values = np.stack(cache["keys"])[first:], np.stack(cache["values"])[first:]
        inverse_root = F32(F32(1.0) / np.sqrt(F32(hd)))
        group = H // KV
        attended = np.zeros(H * hd, dtype=np.float32)
        for h in range(H):
            kv = h // group
            attended[h * hd:(h + 1) * hd] = attend_head_int(
                query_codes[h], F32(query_scales[h] * inverse_root), all_keys[:, kv], np.array(cache["key_scales"][kv][first:], dtype=np.float32),
                all_values[:, kv], np.array(cache["value_scales"][kv][first:], dtype=np.float32))
        gates = np.array([sigmoid(g) for g in gate], dtype=np.float32)
        gated = fake_quantise_int8((attended * gates).astype(np.float32))
        out = a.codebook_matrix(idx("out"))
        return product_rows(out, 0, out[4], gated)

    def push(self, token: int, memory: list | None = None) -> np.ndarray:
        """One token (with a Whistle cross memory: Session::push_with and
        CrossState); returns the lane stream after every layer [layers][lanes·d]."""
        a, lanes, d = self.archive, self.archive.lanes, self.archive.d_model
        self.tokens.append(int(token))
        engram = [self._engram(site, self.position) for site in range(len(a.engram["sites"]))]
        row = self._embedding_row(token)
        stream = np.tile((row * np.sqrt(F32(d))).astype(np.float32), lanes)
        trace = []
        cells = [lane_mean(stream, lanes)]
        for layer in range(a.layers):
            idx = lambda name: self._index(layer, name)  # noqa: E731
            block_input, post, residual = route(self.lane_weights, lanes, layer, layer, stream)
            x = block_input.copy()
            if layer in a.engram["sites"]:  # add_engram (crates/model/src/session.rs:178-188)
                key, value = engram[a.engram["sites"].index(layer)]
                products = (unit_rms(x) * unit_rms(key)).astype(np.float32)
                dot = F32(-0.0)
                for p in products:
                    dot = F32(dot + p)
                alpha = sigmoid(F32(dot / np.sqrt(F32(d))))
                x = (x + (alpha * value).astype(np.float32)).astype(np.float32)
            attended = zero_centred_norm(self._attend(layer, zero_centred_norm(x, a.floats(idx("norm_in")))), a.floats(idx("post_norm")))
            gate = sigmoid(a.floats(idx("attn_gate"))[0])
            x = (x + (gate * attended).astype(np.float32)).astype(np.float32)
            if memory is not None:  # the CrossAttention hook (session.rs:126-128)
                x = cross_apply(a, memory, layer, x, self.heads, self.head_dim)
            mlp = hadamard_apply(a.hadamard(layer), zero_centred_norm(x, a.floats(idx("pre_hada"))))
            x = (x + mlp).astype(np.float32)
            delta = (x - block_input).astype(np.float32)
            mix = residual.reshape(lanes, lanes)
            lanes_in = stream.reshape(lanes, d)
            nxt = np.zeros((lanes, d), dtype=np.float32)
            for lane in range(lanes):
                for source in range(lanes):
                    nxt[lane] = (nxt[lane] + (mix[lane, source] * lanes_in[source]).astype(np.float32)).astype(np.float32)
                nxt[lane] = (nxt[lane] + (post[lane] * delta).astype(np.float32)).astype(np.float32)
            stream = nxt.reshape(-1)
            trace.append(stream.copy())
            cells.append(lane_mean(stream, lanes))
        self.hidden = zero_centred_norm(lane_mean(stream, lanes), self.final_norm)
        for head in self.heads_list:  # ProbeHead::observe of every cell (session.rs:144-147)
            head.observe(cells)
        self.position += 1
        return np.stack(trace)

    def pooled_readout(self, code: int):
        """Session::pooled_readout (session.rs:156-160); None without that head."""
        head = next((h for h in self.heads_list if h.code == code), None)
        return None if head is None else head.pooled()

    def head_output(self, code: int):
        """Session::head_output (session.rs:150-154); None without that head."""
        head = next((h for h in self.heads_list if h.code == code), None)
        return None if head is None else head.project(head.pooled())

    def logits(self) -> np.ndarray:
        """Session::logits (crates/model/src/session.rs:162-175): the fake-quantised
        hidden row through the tied embedding."""
        import struct

        bits, packed, levels, norms, rows, cols = self.embedding
        out_vocab = struct.unpack_from("<48I", self.archive.data, 0)[6]
        return product_int(bits, packed, levels, norms, rows, cols, fake_quantise_int8(self.hidden))[:out_vocab]


# ------------------------------------------------------ Whistle cross attention
_libm.logf.restype = ctypes.c_float
_libm.logf.argtypes = [ctypes.c_float]


def _cross_layer(archive: Archive, layer: int) -> dict:
    """The 10 cross tensors of decoder layer `layer` (crates/cact/src/layout.rs:278-283),
    after the audio manifest that follows the final norm."""
    base = archive.audio_index() + 1 + 10 * layer
    t = {name: base + i for i, name in enumerate(("norm", "q", "k", "v", "gate_proj", "out", "q_norm", "k_norm", "post_norm", "gate"))}
    return t


def cross_memory(archive: Archive, encoded: np.ndarray, heads: int, head_dim: int) -> list:
    """CrossWeights::memory (crates/whistle/src/cross.rs:58-105): each frame
    plus the gated sinusoidal position (angle t · exp(rate · j), rate =
    -ln(10000) / (d/2 - 1); sin in the first half, cos in the second),
    fake-quantised; per layer the key and value products of every frame,
    the keys normed with k_norm, both quantised per (frame, head)."""
    enc = np.asarray(encoded, dtype=np.float32)
    frames, d = enc.shape
    position_gate = archive.floats(archive.audio_index() + 1 + 10 * archive.layers)[0]
    gate = sigmoid(position_gate)
    half = d // 2
    rate = F32(-F32(_libm.logf(10000.0)) / F32(half - 1.0))
    memory = np.zeros((frames, d), dtype=np.float32)
    for t in range(frames):
        out = enc[t].copy()
        for j in range(half):
            angle = F32(F32(t) * F32(_libm.expf(float(F32(rate * F32(j))))))
            out[j] = F32(enc[t, j] + F32(gate * F32(_libm.sinf(float(angle)))))
            out[half + j] = F32(enc[t, half + j] + F32(gate * F32(_libm.cosf(float(angle)))))
        memory[t] = fake_quantise_int8(out)
    layers = []
    for layer in range(archive.layers):
        names = _cross_layer(archive, layer)
        k_proj, v_proj = archive.codebook_matrix(names["k"]), archive.codebook_matrix(names["v"])
        k_norm = archive.floats(names["k_norm"])
        keys = np.zeros((frames, heads, head_dim), dtype=np.int64)
        values = np.zeros_like(keys)
        key_scales = np.zeros((frames, heads), dtype=np.float32)
        value_scales = np.zeros_like(key_scales)
        for t in range(frames):
            k = product_rows(k_proj, 0, k_proj[4], memory[t])
            v = product_rows(v_proj, 0, v_proj[4], memory[t])
            for h in range(heads):
                keys[t, h], key_scales[t, h] = quantise_int8(zero_centred_norm(k[h * head_dim:(h + 1) * head_dim], k_norm))
                values[t, h], value_scales[t, h] = quantise_int8(v[h * head_dim:(h + 1) * head_dim])
        layers.append(dict(keys=keys, key_scales=key_scales, values=values, value_scales=value_scales))
    return layers


def cross_apply(archive: Archive, memory: list, layer: int, x: np.ndarray, heads: int, head_dim: int) -> np.ndarray:
    """CrossState::apply (crates/whistle/src/cross.rs:127-182): the query and
    gate products of the normed, fake-quantised x; per head the normed,
    quantised query; scores dot · key_scale · query_scale over the frames;
    softmax_in_place; the context Σ_frame (value_scale · weight) · code in
    frame order from +0.0; times sigmoid(gate), fake-quantised, the output
    product, post-normed, added with the layer's sigmoid(gate) gain."""
    names = _cross_layer(archive, layer)
    m = memory[layer]
    normed = fake_quantise_int8(zero_centred_norm(x, archive.floats(names["norm"])))
    q = product_rows(archive.codebook_matrix(names["q"]), 0, heads * head_dim, normed)
    gate = product_rows(archive.codebook_matrix(names["gate_proj"]), 0, heads * head_dim, normed)
    q_norm = archive.floats(names["q_norm"])
    inverse_root = F32(F32(1.0) / np.sqrt(F32(head_dim)))
    context = np.zeros(heads * head_dim, dtype=np.float32)
    for h in range(heads):
        codes, scale = quantise_int8(zero_centred_norm(q[h * head_dim:(h + 1) * head_dim], q_norm))
        query_scale = F32(scale * inverse_root)
        dots = (m["keys"][:, h] @ codes).astype(np.float32)
        scores = ((dots * m["key_scales"][:, h]).astype(np.float32) * query_scale).astype(np.float32)
        e = fast_exp((scores - scores.max()).astype(np.float32))
        total = F32(0.0)
        for value in e:
            total = F32(total + value)
        weights = (e * F32(F32(1.0) / total)).astype(np.float32)
        out = np.zeros(head_dim, dtype=np.float32)
        codes_v = m["values"][:, h].astype(np.float32)
        for f in range(weights.size):
            s = F32(m["value_scales"][f, h] * weights[f])
            out = (out + (s * codes_v[f]).astype(np.float32)).astype(np.float32)
        context[h * head_dim:(h + 1) * head_dim] = out
    gates = np.array([sigmoid(g) for g in gate], dtype=np.float32)
    out_proj = archive.codebook_matrix(names["out"])
    attended = product_rows(out_proj, 0, out_proj[4], fake_quantise_int8((context * gates).astype(np.float32)))
    attended = zero_centred_norm(attended, archive.floats(names["post_norm"]))
    gain = sigmoid(archive.floats(names["gate"])[0])
    return (np.asarray(x, dtype=np.float32) + (gain * attended).astype(np.float32)).astype(np.float32)
