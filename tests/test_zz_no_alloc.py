"""nb_model_project_static, the allocation-free codebook product, called
through the C ABI with device buffers and compared bit-exactly with
nb_debug_project (the product with scratch allocated per call) — the tolerance
of every projection test. Collected last so it also runs after the other GPU
tests in one process; it passes alone as well."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STATIC_MAX_TOKENS = 256


@pytest.fixture(scope="module")
def model(native_built, archive_path):
    import rustyneedle_b200 as nb

    return nb.Model.open(archive_path, max_sessions=4)


def _static(model, which, layer, x_dev, out_dev, stream):
    from rustyneedle_b200._native import lib

    fn = lib().nb_model_project_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn(model._h, which, layer, x_dev.data_ptr(), x_dev.shape[0], out_dev.data_ptr(), stream)


def _inputs(seed, tokens):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((tokens, 512)) * rng.uniform(0.01, 3.0, (tokens, 1))).astype(np.float32)


def test_static_product_matches_the_allocating_product_twice_in_a_row(model):
    import torch

    from rustyneedle_b200 import debug

    cases = [(debug.MATRIX_QKVG, 4, 1536, _inputs(70, 40), None),
             (debug.MATRIX_LOGITS, 0, 8192, _inputs(71, 5), torch.cuda.current_stream().cuda_stream)]
    results = []
    for which, layer, rows, x, stream in cases:  # back to back, the second reusing the scratch
        x_dev = torch.from_numpy(x).cuda()
        out_dev = torch.full((x.shape[0], rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        assert _static(model, which, layer, x_dev, out_dev, stream) == 0
        results.append(out_dev.cpu().numpy())
    for (which, layer, rows, x, _), got in zip(cases, results):
        want = debug.project(model, which, layer, x, rows)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (which, layer)


def test_static_product_takes_the_full_scratch_and_rejects_more(model):
    import torch

    from rustyneedle_b200 import debug
    from rustyneedle_b200._native import lib

    x = _inputs(72, STATIC_MAX_TOKENS)
    x_dev = torch.from_numpy(x).cuda()
    out_dev = torch.empty((STATIC_MAX_TOKENS, 512), device="cuda")
    assert _static(model, debug.MATRIX_OUT, 2, x_dev, out_dev, None) == 0
    want = debug.project(model, debug.MATRIX_OUT, 2, x, 512)
    assert np.array_equal(out_dev.cpu().numpy().view(np.uint32), want.view(np.uint32))

    too_many = torch.zeros((STATIC_MAX_TOKENS + 1, 512), device="cuda")
    out_big = torch.empty((STATIC_MAX_TOKENS + 1, 512), device="cuda")
    assert _static(model, debug.MATRIX_OUT, 2, too_many, out_big, None) == -4  # NB_ERR_ARGUMENT
    assert b"static scratch" in lib().nb_last_error()
