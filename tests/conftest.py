"""Shared test configuration.

Markers: ``gpu`` (needs a CUDA device; the CPU run uses ``-m "not gpu"``) and ``slow``.
The ``reference`` fixture makes the reference implementation importable from its offline
install under ``baseline/_ref`` (used as a CPU oracle); tests that need it skip without it.
"""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
REF = ROOT / "baseline" / "_ref"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def reference():
    """Import path of the reference package (CPU oracle)."""
    if not (REF / "nanochat").is_dir():
        pytest.skip("reference install (baseline/_ref) not present")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    import torch
    if not torch.cuda.is_available():
        os.environ.setdefault("NANOCHAT_DTYPE", "float32")
    return REF


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]
