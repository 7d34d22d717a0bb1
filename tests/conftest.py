"""Shared pytest setup: the ``gpu`` marker, the package import and seeded helpers."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

# The reference project's checkout, for the tests that run the reference's own Python
# engine next to this package (LLM_ENGINEERING_REFERENCE overrides the development
# container's read-only mount). GPU boxes have no checkout: those tests skip there.
REFERENCE_ROOT = Path(os.environ.get("LLM_ENGINEERING_REFERENCE", "/root/reference"))

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


@pytest.fixture(scope="session")
def reference_engine():
    """The reference's serving.engine modules, imported from its checkout."""
    if not (REFERENCE_ROOT / "serving" / "engine" / "engine.py").exists():
        pytest.skip("the reference checkout is not available on this machine")
    if str(REFERENCE_ROOT) not in sys.path:
        sys.path.append(str(REFERENCE_ROOT))
    import importlib

    names = ("config", "engine", "request", "paged_kv_storage", "paged_kv_cache",
             "paged_model_runner", "execution", "sequence")
    return {n: importlib.import_module(f"serving.engine.{n}") for n in names}
