"""Shared test configuration.

Markers: ``gpu`` (needs a CUDA device; the CPU run uses ``-m "not gpu"``) and ``slow``.
The ``reference`` fixture makes the reference implementation importable from its offline
install under ``baseline/_ref`` (used as a CPU oracle).  When the install is missing it is made
from the reference's source tree; when neither exists, tests that need it FAIL rather than skip, so
a parity regression cannot hide behind a missing oracle.
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
    from nexttransformer_b200.utils.reference_install import ensure
    try:
        path = ensure(REF)
    except RuntimeError as exc:
        pytest.fail(f"reference install under baseline/_ref failed: {exc}")
    if path is None:
        pytest.fail("reference not installed under baseline/_ref and no source tree to install it from")
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
