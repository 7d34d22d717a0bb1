"""Shared pytest setup: the ``gpu`` marker, the package import and seeded helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def ops():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llm_engineering_b200 import ops as _ops

    return _ops
