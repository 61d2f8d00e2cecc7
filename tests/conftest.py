"""Shared pytest setup: the `gpu` marker, import paths and the built libraries.

Tests marked `gpu` run the sm_100a kernels through the C ABI and compare them
with the CPU oracle (oracle/, a restatement of the reference CPU backend).
Everything else runs on a CPU-only machine.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "random-things_b200", REPO / "oracle", REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import xn_oracle

    xn_oracle.build()
    return xn_oracle


@pytest.fixture(scope="session")
def xn():
    """The product binding; on a GPU run the library must be present and loadable."""
    import xn_fused

    xn_fused.lib()
    return xn_fused


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
