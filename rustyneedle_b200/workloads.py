"""The seeded synthetic workloads of the benchmark configurations.

The reference measures its own weights and tool files only; here every
configuration is a seeded synthetic stand-in with the shapes the benchmark
names. `bench.py` times these workloads and the parity tests decode the same
ones, so the tokens a benchmark run produces are the tokens the tests check
against the CPU restatement.

  config 0  depth 2, batch 1, a 32-token prompt, 64 unconstrained greedy tokens
  config 1  depth 20, batch 1, a 512-token prompt, 256 greedy steps each under
            a seeded bitset allowing ~5 % of the 8192 ids
  config 2  depth 20, 256 sequences per GPU, prompts uniform in [128, 1024]
            (a stratified draw of lengths shared by every rank, order and
            ids seeded per rank: `dp.shard_prompts`), greedy
  config 4  a depth-8 Whistle decoder, 64 utterances, each cross-attending to
            its own 1500 x 512 N(0, 1) encoder output; bos and a language
            token, then 224 greedy text tokens
"""

from __future__ import annotations

import numpy as np

CONFIG0 = dict(depth=2, prompt=32, tokens=64, seed=3)
CONFIG1 = dict(depth=20, prompt=512, steps=256, allowed=0.05, seed=7)
CONFIG2 = dict(depth=20, sequences=256, prompt_low=128, prompt_high=1024, steps=128)
WHISTLE = dict(layers=8, text_vocab=8000, frames=1500, batch=64, tokens=224, seed=11, bos=1)


def config0_prompt() -> np.ndarray:
    rng = np.random.default_rng(CONFIG0["seed"])
    return rng.integers(10, 8000, CONFIG0["prompt"]).astype(np.uint32)


def config1(vocab: int, steps: int | None = None):
    """Config 1's prompt and its per-step grammar bitsets.

    Returns (ids, words, allowed): ids the 512 prompt ids; words[k] the packed
    bitset of step k (vocab/32 uint32 words, bit set = allowed); allowed[k] the
    same set as bool[vocab]. At least one id is allowed every step."""
    rng = np.random.default_rng(CONFIG1["seed"])
    ids = rng.integers(10, 8000, CONFIG1["prompt"]).astype(np.uint32)
    words, allowed = [], []
    for _ in range(CONFIG1["steps"] if steps is None else steps):
        a = rng.random(vocab) < CONFIG1["allowed"]
        a[rng.integers(0, vocab)] = True
        allowed.append(a)
        words.append(np.packbits(a.astype(np.uint8), bitorder="little").view(np.uint32)[: vocab // 32].copy())
    return ids, words, allowed


def config2_prompts(rank: int, count: int = CONFIG2["sequences"]) -> list[np.ndarray]:
    from rustyneedle_b200 import dp

    return dp.shard_prompts(rank, count, CONFIG2["prompt_low"], CONFIG2["prompt_high"])


def whistle_archive():
    """The synthetic Whistle archive of config 4 (depth 8, text vocabulary 8000 of 8192)."""
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=0, geometry=synthetic.Geometry(num_layers=WHISTLE["layers"],
                                                                          text_vocab=WHISTLE["text_vocab"]))


def whistle_encoded(count: int = WHISTLE["batch"], d_model: int = 512):
    """The encoder outputs of config 4's utterances, in order ([frames][d_model] f32 each)."""
    rng = np.random.default_rng(WHISTLE["seed"])
    for _ in range(count):
        yield rng.standard_normal((WHISTLE["frames"], d_model)).astype(np.float32)


def whistle_language(index: int, vocab: int) -> int:
    """The language token utterance `index` is pushed after bos."""
    return WHISTLE["text_vocab"] + index % (vocab - WHISTLE["text_vocab"])


def text_allowed(vocab: int) -> np.ndarray:
    """Whistle::best's restriction to text ids (lib.rs:280-289) as bool[vocab]."""
    a = np.zeros(vocab, dtype=bool)
    a[: WHISTLE["text_vocab"]] = True
    return a


def text_words(vocab: int) -> np.ndarray:
    return np.packbits(text_allowed(vocab), bitorder="little").view(np.uint32)


def token_weight_bytes(depth: int, d: int = 512, heads: int = 8, kv_heads: int = 4, head_dim: int = 64,
                       hada_n: int = 2048, left: int = 64, right: int = 32, rank: int = 8, lanes: int = 4,
                       vocab: int = 8192, group: int = 128, projection_bits: int = 2, embedding_bits: int = 4,
                       phi_bits: int = 4) -> int:
    """Bytes of weights one decode token touches at `depth` layers, in the
    archive's representation (packed codes and fp16 group norms, f32 vectors):
    per layer the q/k/v/gate/out projections, the lane phi rows (4 + 4 + 16 of
    lanes * d columns) and routing scalars, the norms and gates, and the
    Hadamard MLP's diagonals, bias, three Kronecker factor pairs and rank-r
    condition; once per token the two permutations, the final norm, the tied
    logits matrix and one embedding row."""

    def codebook(rows: int, cols: int, bits: int) -> int:
        return rows * cols * bits // 8 + rows * (-(-cols // group)) * 2

    projections = (codebook(heads * head_dim, d, projection_bits) + 2 * codebook(kv_heads * head_dim, d, projection_bits)
                   + codebook(heads * head_dim, d, projection_bits) + codebook(d, heads * head_dim, projection_bits))
    phi = codebook((2 + lanes) * lanes, lanes * d, phi_bits)
    routing = 4 * (3 + 2 * lanes + lanes * lanes)
    vectors = 4 * (d + 2 * head_dim + d + 1 + d)  # norm_in, q_norm, k_norm, post_norm, attn_gate, pre_hada
    hadamard = 4 * (5 * hada_n + 3 * (left * left + right * right) + d * rank + rank * hada_n)
    per_layer = projections + phi + routing + vectors + hadamard
    once = 4 * 2 * hada_n + 4 * d + codebook(vocab, d, embedding_bits) + codebook(1, d, embedding_bits)
    return depth * per_layer + once


def prefill_product_macs(tokens: int, depth: int, d: int = 512, lanes: int = 4, vocab: int = 8192) -> int:
    """int8 multiply-accumulates of the codebook products of a `tokens`-long
    prefill: per token and layer the fused q/k/v/gate (1536 rows), out_proj
    (512 rows) and lane phi rows (24 of lanes * d columns); the logits of the
    last token only."""
    per_token_layer = (1536 + 512) * d + (2 + lanes) * lanes * lanes * d
    return tokens * depth * per_token_layer + vocab * d
