"""Seeded synthetic Needle-3 `.cact` archives.

The reference ships no model files, so every parity case and benchmark in this
repository runs on an archive written here from a seed. The byte format is the
reference's own (a 196-byte header of 48 u32 fields and an f32 rope_theta, the
28-value codebook, 44-byte tensor records, 64-byte aligned blobs; see
crates/cact/src/geometry.rs:41-115, record.rs:38-51, docs/format.md), and the
tensors follow the canonical positional order of crates/cact/src/layout.rs:190-230:
embedding; per layer norm_in, q, k, v, [q, k, v conv taps], q_norm, k_norm, gate_proj, out_proj,
post_norm, attn_gate, pre_hada and 13 Hadamard tensors; nine lane tensors; two
Hadamard permutations; [per engram site: tables, key_proj, value_proj, taps];
final_norm; [the probe-head manifest and each head's probes, gain, query,
row_bias, proj, bias (and calibration for code 3)]; [a Whistle audio section:
manifest, per decoder layer norm, q/k/v/gate/out projections, q_norm, k_norm,
post_norm and gate, the position gate, and one-value placeholders for the
encoder, which this build does not run]; the tokenizer blob.

Weights are codebook-quantised (kind 3): uniform indices, packed least
significant bit first, and one fp16 norm per row drawn log-uniform in
[1e-3, 1e-2] and repeated over the row's 128-column groups. Projections use
2-bit indices; the tied embedding and the lane phi maps use 4-bit indices.
Norm gains are 0.0, so the zero-centred norms apply an effective gain of 1.0.
"""

from __future__ import annotations

import hashlib
import os
import struct
import tempfile
from dataclasses import dataclass, field

import numpy as np

FORMAT_TAG = 0x05E12A84
HEADER_BYTES = 196
RECORD_BYTES = 44
ALIGN = 64

KIND_HALF, KIND_SINGLE, KIND_CODEBOOK, KIND_RAW = 1, 2, 3, 4

# Lloyd-Max levels of a unit Gaussian (2, 3 and 4 bits); the archive stores them
# divided by sqrt(group) so that a unit-norm group maps onto them.
_LLOYD_MAX = {
    2: [0.4528, 1.5104],
    3: [0.2451, 0.7560, 1.3440, 2.1520],
    4: [0.1284, 0.3881, 0.6568, 0.9424, 1.2562, 1.6181, 2.0690, 2.7326],
}


@dataclass
class Geometry:
    vocab: int = 8192
    out_vocab: int = 8192
    d_model: int = 512
    num_heads: int = 8
    num_kv_heads: int = 4
    num_layers: int = 20
    head_dim: int = 64
    max_seq_len: int = 2048
    hada_n: int = 2048
    hada_left: int = 64
    hada_right: int = 32
    lanes: int = 4
    rope_theta: float = 10000.0
    group: int = 128
    projection_bits: int = 2
    embedding_bits: int = 4
    phi_bits: int = 4
    rank: int = 8
    # optional Needle-3 features (0 = absent; the defaults write none of them)
    sliding_window: int = 0   # window of the non-global layers
    global_layers: int = 0    # bit l set: layer l attends to the whole context
    conv_taps: int = 0        # causal convolution taps on q, k and v
    engram_sites: tuple = ()  # layers that add the hashed n-gram memory
    engram_slots: int = 4096  # rows per table
    engram_sub_dim: int = 128
    engram_orders: tuple = (2, 3)
    engram_heads_per_order: int = 2
    engram_conv_taps: int = 3
    engram_dilation: int = 2
    engram_seed_heads: int = 0
    probe_heads: tuple = ()   # head manifest codes (1, 2 or 3)
    probes_per_layer: int = 2
    head_queries: int = 2
    head_outputs: int = 3
    text_vocab: int = 0       # > 0: a Whistle archive (audio manifest, cross-attention tensors per decoder layer)
    extra: dict = field(default_factory=dict)


def _codebook(rng: np.random.Generator, group: int) -> np.ndarray:
    out = []
    for bits in (2, 3, 4):
        half = np.array(_LLOYD_MAX[bits], dtype=np.float64)
        half = half * (1.0 + 0.01 * rng.standard_normal(half.shape))
        half = np.sort(np.abs(half))
        levels = np.concatenate([-half[::-1], half]) / np.sqrt(group)
        out.append(levels.astype(np.float32))
    return np.concatenate(out)


class _Writer:
    def __init__(self) -> None:
        self.records: list[tuple] = []
        self.blobs: list[bytes] = []

    def add(self, kind: int, shape: tuple, blob: bytes, group: int = 0, bits: int = 0) -> int:
        self.records.append((kind, tuple(shape), len(blob), group, bits))
        self.blobs.append(blob)
        return len(self.records) - 1

    def single(self, values: np.ndarray) -> int:
        values = np.asarray(values, dtype=np.float32)
        return self.add(KIND_SINGLE, values.shape, values.tobytes())

    def codebook_matrix(self, rng: np.random.Generator, rows: int, columns: int, bits: int, group: int) -> int:
        packed, norms = _codebook_rows(rng, rows, columns, bits, group)
        return self.add(KIND_CODEBOOK, (rows, columns), packed.tobytes() + norms.tobytes(), group, bits)

    def finish(self, path: str, header_fields: list[int], rope_theta: float, codebook: np.ndarray) -> None:
        directory_at = HEADER_BYTES + codebook.size * 4
        offset = directory_at + RECORD_BYTES * len(self.records)
        offsets = []
        for blob in self.blobs:
            offset = -(-offset // ALIGN) * ALIGN
            offsets.append(offset)
            offset += len(blob)
        with open(path, "wb") as f:
            f.write(struct.pack("<48I", *header_fields))
            f.write(struct.pack("<f", rope_theta))
            f.write(codebook.astype("<f4").tobytes())
            for (kind, shape, nbytes, group, bits), at in zip(self.records, offsets):
                dims = list(shape) + [0] * (4 - len(shape))
                f.write(struct.pack("<BBH4IQQII", kind, len(shape), 0, *dims, at, nbytes, group, bits))
            position = directory_at + RECORD_BYTES * len(self.records)
            for blob, at in zip(self.blobs, offsets):
                f.write(b"\0" * (at - position))
                f.write(blob)
                position = at + len(blob)


def _codebook_rows(rng: np.random.Generator, rows: int, columns: int, bits: int, group: int):
    """The draws of _Writer.codebook_matrix: packed indices and fp16 norms (as uint16)."""
    padded = -(-columns // group) * group
    groups = padded // group
    packed = rng.integers(0, 256, size=rows * padded * bits // 8, dtype=np.uint8)
    norm = np.exp(rng.uniform(np.log(1e-3), np.log(1e-2), size=rows)).astype(np.float16)
    return packed, np.repeat(norm, groups).view(np.uint16)


def _levels(codebook: np.ndarray, bits: int) -> np.ndarray:
    start = {2: 0, 3: 4, 4: 12}[bits]
    return codebook[start:start + (1 << bits)].copy()


def embedding_raw(seed: int = 0, geometry: Geometry | None = None):
    """The embedding tensor of write_archive(seed, geometry) in the archive's
    representation: (packed indices, codebook levels, fp16 norms as uint16)."""
    g = geometry or Geometry()
    rng = np.random.default_rng(seed)
    codebook = _codebook(rng, g.group)
    packed, norms = _codebook_rows(rng, g.vocab, g.d_model, g.embedding_bits, g.group)
    return packed, _levels(codebook, g.embedding_bits), norms


def product_matrix(seed: int, rows: int, columns: int, bits: int, group: int = 128):
    """A codebook-quantised matrix for the product microbenchmark, drawn like
    the archive's: Lloyd-Max-shaped levels, uniform indices, one log-uniform
    [1e-3, 1e-2] fp16 norm per row repeated over its groups. Returns (packed
    indices, levels, fp16 norms as uint16)."""
    rng = np.random.default_rng(seed)
    codebook = _codebook(rng, group)
    packed, norms = _codebook_rows(rng, rows, columns, bits, group)
    return packed, _levels(codebook, bits), norms


def tokenizer_blob(vocab: int) -> bytes:
    """A minimal valid vocabulary blob (crates/tokenizer/src/vocabulary.rs:66-99):
    specials, the 256 byte pieces, then filler pieces up to `vocab`."""
    specials = [("<unk>", 1), ("<s>", 2), ("</s>", 2), ("<pad>", 2), ("<|im_start|>", 3), ("<|im_end|>", 3),
                ("<think>", 3), ("</think>", 3), ("<tool_call>", 3), ("</tool_call>", 3)]
    pieces = specials + [(f"<0x{b:02X}>", 4) for b in range(256)]
    while len(pieces) < vocab:
        pieces.append((f"▁t{len(pieces)}", 0))
    pieces = pieces[:vocab]
    out = bytearray(struct.pack("<5IBBH", len(pieces), 3, 2, 1, 0, 1, 1, 0))
    for index, (text, kind) in enumerate(pieces):
        raw = text.encode()
        out += struct.pack("<fBH", -float(index), kind, len(raw)) + raw
    return bytes(out)


def write_archive(path: str, seed: int = 0, geometry: Geometry | None = None) -> str:
    """Writes a synthetic Needle-3 archive and returns its path."""
    g = geometry or Geometry()
    rng = np.random.default_rng(seed)
    codebook = _codebook(rng, g.group)
    w = _Writer()
    d, hd, H, KV, L, n = g.d_model, g.head_dim, g.num_heads, g.num_kv_heads, g.num_layers, g.hada_n
    zeros = lambda count: np.zeros(count, dtype=np.float32)  # noqa: E731

    w.codebook_matrix(rng, g.vocab, d, g.embedding_bits, g.group)
    for _ in range(L):
        w.single(zeros(d))  # norm_in
        w.codebook_matrix(rng, H * hd, d, g.projection_bits, g.group)  # q
        w.codebook_matrix(rng, KV * hd, d, g.projection_bits, g.group)  # k
        w.codebook_matrix(rng, KV * hd, d, g.projection_bits, g.group)  # v
        if g.conv_taps > 0:  # q, k, v taps [tap][width]: tap 0 near 1, older taps smaller
            for width in (H * hd, KV * hd, KV * hd):
                if g.extra.get("identity_taps"):  # tap 0 = 1, the rest 0, drawing nothing
                    taps = np.zeros((g.conv_taps, width))
                    taps[0] = 1.0
                else:
                    taps = 0.3 * rng.standard_normal((g.conv_taps, width))
                    taps[0] += 1.0
                w.single(taps)
        w.single(zeros(hd))  # q_norm
        w.single(zeros(hd))  # k_norm
        w.codebook_matrix(rng, H * hd, d, g.projection_bits, g.group)  # gate_proj
        w.codebook_matrix(rng, d, H * hd, g.projection_bits, g.group)  # out_proj
        w.single(zeros(d))  # post_norm
        w.single(rng.standard_normal(1))  # attn_gate
        w.single(zeros(d))  # pre_hada
        w.single(rng.standard_normal(n))  # d1
        w.single(rng.standard_normal(n))  # d2
        w.single(0.1 * rng.standard_normal(n))  # b2
        w.single(rng.standard_normal(n))  # d3
        w.single(rng.standard_normal(n))  # d4
        for _ in range(3):  # w?a (left) and w?b (right) Kronecker factors
            w.single(rng.standard_normal((g.hada_left, g.hada_left)) / np.sqrt(g.hada_left))
            w.single(rng.standard_normal((g.hada_right, g.hada_right)) / np.sqrt(g.hada_right))
        w.single(rng.standard_normal((d, g.rank)) / np.sqrt(d))  # cond_v
        w.single(0.1 * rng.standard_normal((g.rank, n)))  # cond_u
    lanes = g.lanes
    w.single(rng.standard_normal(L))  # a_pre
    w.single(rng.standard_normal(L))  # a_post
    w.single(rng.standard_normal(L))  # a_res
    w.single(rng.standard_normal(L * lanes))  # b_pre
    w.single(rng.standard_normal(L * lanes))  # b_post
    w.single(rng.standard_normal(L * lanes * lanes))  # b_res
    w.codebook_matrix(rng, L * lanes, lanes * d, g.phi_bits, g.group)  # phi_pre
    w.codebook_matrix(rng, L * lanes, lanes * d, g.phi_bits, g.group)  # phi_post
    w.codebook_matrix(rng, L * lanes * lanes, lanes * d, g.phi_bits, g.group)  # phi_res
    w.single(rng.permutation(n).astype(np.float32))
    w.single(rng.permutation(n).astype(np.float32))
    tables = len(g.engram_orders) * g.engram_heads_per_order
    for _ in g.engram_sites:  # crates/cact/src/layout.rs:231-234: tables, key_proj, value_proj, taps
        w.codebook_matrix(rng, tables * g.engram_slots, g.engram_sub_dim, g.projection_bits, g.group)
        w.codebook_matrix(rng, d, tables * g.engram_sub_dim, g.projection_bits, g.group)
        w.codebook_matrix(rng, d, tables * g.engram_sub_dim, g.projection_bits, g.group)
        if g.extra.get("zero_engram_taps"):  # the value convolution adds nothing, drawing nothing
            w.single(np.zeros((g.engram_conv_taps, d)))
        else:
            taps = 0.5 * rng.standard_normal((g.engram_conv_taps, d))
            taps[0] += 1.0
            w.single(taps)
    w.single(zeros(d))  # final_norm
    if g.probe_heads:  # crates/cact/src/layout.rs:236-254: manifest, then per head 6 tensors (+ calibration for code 3)
        w.add(KIND_HALF, (len(g.probe_heads),), np.array(g.probe_heads, dtype=np.float16).tobytes())
        slots = (L + 1) * g.probes_per_layer
        for code in g.probe_heads:
            w.codebook_matrix(rng, slots, d, g.embedding_bits, g.group)  # probes
            w.single(1.0 + 0.1 * rng.standard_normal(slots))  # gain
            w.codebook_matrix(rng, g.head_queries, d, g.embedding_bits, g.group)  # query
            w.single(0.5 * rng.standard_normal(g.head_queries * slots))  # row_bias
            w.codebook_matrix(rng, g.head_outputs, g.head_queries * d, g.projection_bits, g.group)  # proj
            w.single(0.1 * rng.standard_normal(g.head_outputs))  # bias
            if code == 3:
                w.single(rng.standard_normal(4))  # calibration
    if g.text_vocab:  # crates/cact/src/layout.rs:256-293: manifest, 10 cross tensors per decoder layer, position gate, encoder
        # manifest: magic, version, text_vocab, encoder_layers, encoder_lanes, conv_kernel, stem_channels, stem_stages,
        # mels, sample_rate, fft_size, window, hop. The encoder is not part of this build: no encoder layers, one stem
        # stage, and one-value placeholders for its lanes, final norm, stem and mel tensors.
        w.single(np.array([3246, 1, g.text_vocab, 0, lanes, 31, 64, 1, 80, 16000, 400, 400, 160], dtype=np.float32))
        for _ in range(L):
            w.single(zeros(d))  # norm
            for _ in range(4):  # q, k, v, gate projections
                w.codebook_matrix(rng, H * hd, d, g.projection_bits, g.group)
            w.codebook_matrix(rng, d, H * hd, g.projection_bits, g.group)  # out_proj
            w.single(zeros(hd))  # q_norm
            w.single(zeros(hd))  # k_norm
            w.single(zeros(d))  # post_norm
            w.single(rng.standard_normal(1))  # gate
        w.single(rng.standard_normal(1))  # position gate
        for _ in range(9 + 1 + 1 + 1 + 1):  # encoder lanes, final norm, stem first and out, mel
            w.single(zeros(1))
    w.add(KIND_RAW, (0,), tokenizer_blob(g.vocab))

    header = [FORMAT_TAG, len(w.records), codebook.size, 0, 8, g.vocab, g.out_vocab, d, H, KV, L, hd, hd,
              g.max_seq_len, n, lanes, g.sliding_window, g.global_layers & 0xFFFFFFFF, g.global_layers >> 32, g.conv_taps]
    if g.engram_sites:
        orders = list(g.engram_orders) + [0] * (4 - len(g.engram_orders))
        sites = list(g.engram_sites) + [0] * (16 - len(g.engram_sites))
        header += [g.engram_slots, g.engram_sub_dim, tables, g.engram_conv_taps, g.engram_dilation, g.engram_seed_heads,
                   len(g.engram_orders)] + orders + [len(g.engram_sites)] + sites
    else:
        header += [0] * 28
    assert len(header) == 48
    w.finish(path, header, g.rope_theta, codebook)
    return path


def cached_archive(seed: int = 0, geometry: Geometry | None = None, directory: str | None = None) -> str:
    """The path of a synthetic archive for (seed, geometry), written once per machine."""
    g = geometry or Geometry()
    key = hashlib.sha1(repr((seed, sorted(vars(g).items()))).encode()).hexdigest()[:16]
    directory = directory or os.environ.get("NEEDLE_B200_CACHE", os.path.join(tempfile.gettempdir(), "needle_b200"))
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"synthetic_{seed}_{key}.cact")
    if not os.path.exists(path):
        partial = f"{path}.{os.getpid()}.partial"
        write_archive(partial, seed, g)
        os.replace(partial, path)
    return path
