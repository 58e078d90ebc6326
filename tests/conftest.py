"""Test configuration.

- `-m "not gpu"` (this container, no GPU): the oracle against the reference's golden vectors, the
  host-side logic of the Python mirror, and that the C-ABI library loads and exports every symbol
  its header declares.
- `-m gpu` (a B200): parity of every CUDA kernel, called through the C-ABI, against the oracle.

Seeds are fixed per test like the reference's suite (`tests/conftest.py:31-33` of the reference).
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "llm-decode-kernels_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); skipped without one")
    config.addinivalue_line("markers", "slow: large shapes")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


ON_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    skip_gpu = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords and not ON_GPU:
            item.add_marker(skip_gpu)


@pytest.fixture(autouse=True)
def _seed():
    np.random.seed(0)
    try:
        import torch

        torch.manual_seed(0)
    except Exception:
        pass


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / f"{name}.npz"))
        return cache[name]

    return load


os.environ.setdefault("DECODEK_STRICT", "1")
