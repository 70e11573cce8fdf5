"""Compute dtype: ``NANOCHAT_DTYPE`` (bfloat16 | float16 | float32) or bf16 on CUDA, fp32 on CPU.

Master weights stay fp32; activations and matmuls run in the compute dtype (no autocast).
Same rule as the reference's ``nanochat/common.py:17-33``.
"""
import os

import torch

_NAMES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _detect():
    env = os.environ.get("NANOCHAT_DTYPE")
    if env:
        return _NAMES[env]
    if torch.cuda.is_available() and torch.cuda.get_device_capability() >= (8, 0):
        return torch.bfloat16
    return torch.float32


COMPUTE_DTYPE = _detect()
