"""Shared fixtures. CPU tests (-m "not gpu") exercise the oracle, the archive
writer and the C-ABI library's loading and error paths; GPU tests (-m gpu)
compare the sm_100a kernels with the oracle through the C ABI."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def archive_path():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=0)


@pytest.fixture(scope="session")
def small_archive_path():
    """A 4-layer archive of the same geometry (fast oracle runs)."""
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=1, geometry=synthetic.Geometry(num_layers=4))


@pytest.fixture(scope="session")
def native_built():
    from rustyneedle_b200 import build

    return build.build()


def prompt_ids(seed: int, count: int, low: int = 10, high: int = 8000) -> np.ndarray:
    return np.random.default_rng(seed).integers(low, high, count).astype(np.uint32)


def random_mask(rng: np.random.Generator, vocab: int, p: float = 0.05) -> np.ndarray:
    """A packed allowed-token bitset (bit set = allowed), at least one id allowed."""
    allowed = rng.random(vocab) < p
    if not allowed.any():
        allowed[rng.integers(0, vocab)] = True
    return np.packbits(allowed.astype(np.uint8), bitorder="little").view(np.uint32), allowed
