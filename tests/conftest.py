"""Shared fixtures. GPU tests are marked ``gpu`` and skipped without CUDA."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def native_lib():
    """The in-tree native library, built if missing (never a CPU fallback)."""
    from zipserv_asplos26_b200 import build, runtime

    if not runtime.library_path().is_file():
        if os.environ.get("ZIPSERV_LIBRARY"):
            pytest.fail("ZIPSERV_LIBRARY points at a missing library")
        build.build()
    runtime._library.cache_clear()
    return runtime._library()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle

    oracle.ensure_built()
    return oracle
