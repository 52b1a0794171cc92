"""Shared fixtures.

Tests that need a B200 are marked ``gpu`` and are selected with ``-m gpu``; the
CPU suite (``-m "not gpu"``) covers the oracle against the golden fixtures, the
host-side logic, and that the C-ABI library loads and exports every symbol the
header declares.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    # A gpu-marked test selected on a machine without a GPU fails loudly rather
    # than skipping: a silent skip would read as a pass.
    return None


@pytest.fixture(autouse=True)
def deterministic_seed() -> None:
    torch.manual_seed(0)


@pytest.fixture(scope="session")
def cuda_device() -> torch.device:
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert major == 10, f"gpu tests need an sm_100 device, got sm_{major}{minor}"
    return torch.device("cuda", 0)
