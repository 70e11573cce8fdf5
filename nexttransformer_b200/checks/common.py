"""Helpers shared by the checks: source digest and parameter digest."""
import hashlib
from pathlib import Path

import torch

PACKAGE = Path(__file__).resolve().parents[1]


def source_hash():
    """sha256 over the package's Python and CUDA/C++ sources (path + bytes, sorted)."""
    h = hashlib.sha256()
    files = sorted(p for p in PACKAGE.rglob("*") if p.suffix in (".py", ".cu", ".cuh", ".cpp", ".h")
                   and "__pycache__" not in p.parts)
    for p in files:
        h.update(p.relative_to(PACKAGE.parent).as_posix().encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def parameter_digest(model):
    h = hashlib.sha256()
    for name, p in model.named_parameters():
        h.update(name.encode())
        h.update(p.detach().contiguous().view(torch.uint8).cpu().numpy().tobytes())
    return h.hexdigest()
