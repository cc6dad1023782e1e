"""Shared pytest configuration: the `gpu` marker, import paths, fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built libh3b.so")


@pytest.fixture(scope="session")
def ref():
    """The reference's own Python modules, or skip when the tree is absent."""
    from oracle import reference

    r = reference.load()
    if r is None:
        pytest.skip("reference tree not present (expected on GPU boxes)")
    return r


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from minixmax_h3_b200 import _lib

    _lib.lib()  # must load: no silent fallback
    return torch.device("cuda", 0)
