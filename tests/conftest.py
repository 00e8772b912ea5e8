"""Test configuration: import paths, the `gpu` marker, shared fixtures.

`-m "not gpu"` runs on any machine: the oracle against the reference's golden vectors, the
host-side logic (block tables, round bookkeeping, request sharding over gloo ranks) and a
check that libspecb200.so loads and exports every symbol include/specb200.h declares.
`-m gpu` runs the CUDA path through the C ABI against the oracle and the golden vectors.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "speculative-decoder_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a kernels)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_accept() -> dict:
    return dict(np.load(GOLDEN / "accept.npz"))


@pytest.fixture(scope="session")
def golden_forward() -> dict:
    return dict(np.load(GOLDEN / "forward.npz"))


@pytest.fixture(scope="session")
def golden_ngram() -> list:
    return json.loads((GOLDEN / "ngram.json").read_text())


@pytest.fixture(scope="session")
def golden_paged() -> dict:
    return json.loads((GOLDEN / "paged.json").read_text())


@pytest.fixture(scope="session")
def golden_generate() -> dict:
    return json.loads((GOLDEN / "generate.json").read_text())


def random_prompts(n: int, vocab: int, seed: int, low: int = 3, high: int = 20) -> list[list[int]]:
    """Same recipe as the reference's tests/conftest.py:36-39."""
    gen = torch.Generator().manual_seed(seed)
    lengths = torch.randint(low, high, (n,), generator=gen).tolist()
    return [torch.randint(0, vocab, (m,), generator=gen).tolist() for m in lengths]


def tiny_fp32(seed: int = 0):
    """The reference's tiny fixture (lm/load.py:124-141, seed 0): weights drawn in fp32, so
    the fp64 reference and the fp32 engine hold identical values."""
    from lm.load import tiny_model

    return tiny_model(seed=seed, dtype=torch.float32)


def early_exit(model, n_layers: int = 1):
    """The target truncated to its first layers (tests/conftest.py:20-28 of the reference)."""
    import copy

    draft = copy.deepcopy(model)
    draft.model.layers = draft.model.layers[:n_layers]
    draft.config.num_hidden_layers = n_layers
    return draft
