"""NVTX ranges for step timelines (Nsight Systems, ncu's range filters).

``NT_NVTX=1`` in the environment turns them on; otherwise ``nvtx_range`` is a no-op context manager
and costs one attribute lookup.  Ranges mark the training step, each micro-batch, each layer's
forward and backward, the head, the optimizer phases and every collective issue point, so a step
timeline can be attributed without a kernel profiler.
"""
import os
from contextlib import contextmanager

ENABLED = os.environ.get("NT_NVTX", "0") == "1"


@contextmanager
def _range(name):
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NULL = _Null()


def nvtx_range(name):
    """Context manager marking ``name`` on the NVTX timeline when ``NT_NVTX=1``."""
    return _range(name) if ENABLED else _NULL
