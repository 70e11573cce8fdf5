"""Process bootstrap: one process per GPU, ``torch.distributed`` over NCCL (gloo on CPU).

``initialize(seed)`` reads WORLD_SIZE / RANK / LOCAL_RANK, binds the device, creates the
process group with a bounded timeout and seeds every RNG (reference behaviour:
``nexttransformer/runtime/process.py:16-29``).
"""
from datetime import timedelta
import json
import os
from pathlib import Path
import random
import time

import numpy as np
import torch
import torch.distributed as dist


def initialize(seed=42, timeout_s=600):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
        torch.backends.cuda.matmul.allow_tf32 = True
        torch.backends.cudnn.allow_tf32 = True
    if world > 1 and not dist.is_initialized():
        kw = dict(backend="nccl" if device.type == "cuda" else "gloo", timeout=timedelta(seconds=timeout_s))
        if device.type == "cuda":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if device.type == "cuda":
        torch.cuda.manual_seed_all(seed)
    return rank, world, device


def synchronize(device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def reduce_sum(t):
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t)
    return t


def reduce_max(t):
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t


def append_event(output, event):
    with (Path(output) / "metrics.jsonl").open("a") as f:
        f.write(json.dumps(event, ensure_ascii=False) + "\n")


def rng_state():
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}


def restore_rng(state):
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"])
    if state.get("cuda") is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(state["cuda"])


def shutdown():
    if dist.is_initialized():
        dist.destroy_process_group()
