"""The product microbenchmark's shapes (K, N) in {(512, 2048), (2048, 512),
(512, 8192)} at several token counts, through the C ABI hook
nb_debug_product, bit-exact against the CPU restatement's INT product
(QuantisedMatrix::prepare + multiply_vector, crates/kernels/src/matrix.rs:123-165).
Token counts cover the CUDA-core GEMV (<= 8), the 16-token and 32-token
tensor-core tiles, large passes with a ragged last block (600 and 2100
tokens), and K = 2048 (four 512-column chunks)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(512, 2048, 2), (2048, 512, 2), (2048, 512, 4), (512, 8192, 4)]


@pytest.mark.parametrize("cols,rows,bits", SHAPES)
@pytest.mark.parametrize("tokens", [1, 8, 13, 40, 256, 600, 2100])
def test_product_matches_the_integer_restatement(native_built, oracle_lib, cols, rows, bits, tokens):
    from rustyneedle_b200 import debug, synthetic

    packed, levels, norms = synthetic.product_matrix(seed=cols + rows + bits, rows=rows, columns=cols, bits=bits)
    rng = np.random.default_rng(tokens)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 3.0, (tokens, 1))).astype(np.float32)
    if tokens > 1:
        x[-1] = 0.0  # an all-zero input: every group scale falls back to 1
    got, _ = debug.product(bits, packed, levels, norms, rows, cols, x)
    for t in sorted({0, tokens // 2, tokens - 1}):
        want = oracle_lib.product_raw(oracle_lib.MODE_INT, bits, packed, levels, norms, rows, cols, x[t])
        assert np.array_equal(got[t].view(np.uint32), want.view(np.uint32)), (t, np.flatnonzero(got[t] != want)[:5])


def test_product_timing_is_reported(native_built):
    from rustyneedle_b200 import debug, synthetic

    packed, levels, norms = synthetic.product_matrix(seed=1, rows=2048, columns=512, bits=2)
    x = np.random.default_rng(0).standard_normal((64, 512)).astype(np.float32)
    _, ms = debug.product(2, packed, levels, norms, 2048, 512, x, reps=5)
    assert 0.0 < ms < 50.0


@pytest.mark.parametrize("cols,rows,bits", [(512, 2048, 2), (512, 8192, 4), (512, 512, 2)])
@pytest.mark.parametrize("tokens", [256, 300, 449, 1000])
def test_large_pass_product_every_token(native_built, oracle_lib, cols, rows, bits, tokens):
    """Passes of at least 256 tokens through a K = 512 matrix run the
    persistent, pipelined tensor-core product (64-token tiles, two TMEM
    accumulator sets, TMA tensor stores of whole 8-token chunks and plain
    stores where a warp's tokens run past the pass): every token's row of
    outputs, ragged last tiles (300 = 4·64 + 44, 449 = 7·64 + 1) and CTAs that
    walk several tiles included, bit-exact against the restatement."""
    from rustyneedle_b200 import debug, synthetic

    packed, levels, norms = synthetic.product_matrix(seed=3 * cols + rows + bits, rows=rows, columns=cols, bits=bits)
    rng = np.random.default_rng(tokens + rows)
    x = (rng.standard_normal((tokens, cols)) * rng.uniform(0.01, 3.0, (tokens, 1))).astype(np.float32)
    x[tokens // 3] = 0.0
    got, _ = debug.product(bits, packed, levels, norms, rows, cols, x)
    for t in range(tokens):
        want = oracle_lib.product_raw(oracle_lib.MODE_INT, bits, packed, levels, norms, rows, cols, x[t])
        assert np.array_equal(got[t].view(np.uint32), want.view(np.uint32)), (t, np.flatnonzero(got[t] != want)[:5])
