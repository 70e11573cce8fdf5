"""Checkpoints in both formats of the reference.

Formal format (``nexttransformer/runtime/checkpoint.py``): ``checkpoint_%08d/`` holding
``model.pt`` {model, model_config, train_config, state, world_size} (rank 0),
``rank_%04d.pt`` {optimizer, rng, data, routing_rng} per rank and ``complete.json``
{step, world_size, files: {name: {bytes, sha256}}}; ``latest.json`` points at the newest.
Every file is written to a temporary name and renamed; barriers order the phases, and the
completion marker appears only when every shard is on disk.

nanochat format (``nanochat/checkpoint_manager.py``): ``model_%06d.pt`` (state dict),
``optim_%06d_rank%d.pt`` per rank and ``meta_%06d.json``.

Models trained on the fused path keep fp32 gradients outside autograd; that state is not
checkpointed (gradients are recomputed every update), only parameters and optimizer state.
"""
from dataclasses import asdict, is_dataclass
import json
import os
from pathlib import Path
import shutil

import torch
import torch.distributed as dist

from nexttransformer_b200.runtime.files import atomic_json, sha256
from nexttransformer_b200.runtime.process import restore_rng, rng_state


def _barrier(world):
    if world > 1 and dist.is_initialized():
        dist.barrier()


def _cfg(x):
    return asdict(x) if is_dataclass(x) else x


def save_checkpoint(output, model, optimizer, stream, mc, tc, state, rank=0, world=1):
    directory = Path(output) / f"checkpoint_{state['step']:08d}"
    if rank == 0:
        directory.mkdir(parents=True, exist_ok=False)
    _barrier(world)
    tmp = directory / f"rank_{rank:04d}.pt.tmp"
    routing = model.routing_rng_state() if hasattr(model, "routing_rng_state") else None
    torch.save({"optimizer": optimizer.state_dict() if optimizer is not None else None, "rng": rng_state(),
                "data": stream.state_dict() if stream is not None else None, "routing_rng": routing}, tmp)
    tmp.replace(directory / f"rank_{rank:04d}.pt")
    if rank == 0:
        tmp = directory / "model.pt.tmp"
        torch.save({"model": model.state_dict(), "model_config": _cfg(mc), "train_config": _cfg(tc), "state": state,
                    "world_size": world}, tmp)
        tmp.replace(directory / "model.pt")
    _barrier(world)
    if rank == 0:
        files = {p.name: {"bytes": p.stat().st_size, "sha256": sha256(p)} for p in sorted(directory.glob("*.pt"))}
        atomic_json(directory / "complete.json", {"step": state["step"], "world_size": world, "files": files})
        atomic_json(Path(output) / "latest.json", {"step": state["step"], "checkpoint": directory.name})
    _barrier(world)
    return directory


def verify_checkpoint(path, names):
    manifest = json.loads((Path(path) / "complete.json").read_text())
    for name in names:
        item = manifest["files"][name]
        p = Path(path) / name
        if p.stat().st_size != item["bytes"] or sha256(p) != item["sha256"]:
            raise ValueError(f"checkpoint checksum mismatch: {name}")
    return manifest


def load_optimizer_state(optimizer, state_dict):
    """``optimizer.load_state_dict`` that keeps the saved dtype of every floating state tensor.
    torch casts each parameter's state to the parameter's dtype on load; the update kernels keep fp32
    moments for the bf16 embedding tables, so those are restored from the saved fp32 tensors."""
    optimizer.load_state_dict(state_dict)
    params = [p for group in optimizer.param_groups for p in group["params"]]
    for index, saved in state_dict["state"].items():
        live = optimizer.state[params[index]]
        for key, value in saved.items():
            if torch.is_tensor(value) and value.is_floating_point() and live[key].dtype != value.dtype:
                live[key] = value.to(device=params[index].device)


def load_checkpoint(path, model, optimizer=None, stream=None, rank=0, world=1):
    path = Path(path)
    manifest = json.loads((path / "complete.json").read_text())
    if optimizer is not None and manifest["world_size"] != world:
        raise ValueError("optimizer and data sharding require the original world size")
    verify_checkpoint(path, ["model.pt"] + ([f"rank_{rank:04d}.pt"] if optimizer is not None else []))
    saved = torch.load(path / "model.pt", map_location="cpu", weights_only=False)
    model.load_state_dict(saved["model"], strict=True)
    if hasattr(model, "refresh_shadows"):
        model.refresh_shadows()
    if optimizer is not None:
        local = torch.load(path / f"rank_{rank:04d}.pt", map_location="cpu", weights_only=False)
        load_optimizer_state(optimizer, local["optimizer"])
        if stream is not None and local["data"] is not None:
            stream.load_state_dict(local["data"])
        restore_rng(local["rng"])
        if local.get("routing_rng") is not None and hasattr(model, "restore_routing_rng"):
            model.restore_routing_rng(local["routing_rng"])
    return saved


def complete_checkpoints(output):
    """Steps of checkpoints whose completion marker exists, ascending."""
    out = []
    for d in Path(output).glob("checkpoint_*"):
        if (d / "complete.json").exists():
            out.append(int(d.name.split("_")[1]))
    return sorted(out)


def set_aside_incomplete(output):
    """Move checkpoint directories without a completion marker to incomplete_checkpoints/."""
    moved = []
    for d in sorted(Path(output).glob("checkpoint_*")):
        if not (d / "complete.json").exists():
            dest = Path(output) / "incomplete_checkpoints" / d.name
            dest.parent.mkdir(parents=True, exist_ok=True)
            shutil.move(str(d), str(dest))
            moved.append(d.name)
    return moved


def prune_rolling(output, keep, protected=()):
    """Keep the newest `keep` rolling checkpoints; protocol checkpoints (protected steps) stay."""
    steps = [s for s in complete_checkpoints(output) if s not in set(protected)]
    for s in steps[:-keep] if keep > 0 else steps:
        shutil.rmtree(Path(output) / f"checkpoint_{s:08d}", ignore_errors=True)


# ------------------------------------------------------------------ nanochat format
def save_nanochat(checkpoint_dir, step, model_data, optimizer_data, meta_data, rank=0):
    os.makedirs(checkpoint_dir, exist_ok=True)
    if rank == 0:
        torch.save(model_data, os.path.join(checkpoint_dir, f"model_{step:06d}.pt"))
        atomic_json(os.path.join(checkpoint_dir, f"meta_{step:06d}.json"), meta_data)
    if optimizer_data is not None:
        torch.save(optimizer_data, os.path.join(checkpoint_dir, f"optim_{step:06d}_rank{rank:d}.pt"))


def load_nanochat(checkpoint_dir, step, device="cpu", load_optimizer=False, rank=0):
    model = torch.load(os.path.join(checkpoint_dir, f"model_{step:06d}.pt"), map_location=device)
    opt = None
    if load_optimizer:
        opt = torch.load(os.path.join(checkpoint_dir, f"optim_{step:06d}_rank{rank:d}.pt"), map_location=device)
    meta = json.loads(Path(checkpoint_dir, f"meta_{step:06d}.json").read_text())
    return model, opt, meta


def last_nanochat_step(checkpoint_dir):
    steps = [int(p.stem.split("_")[1]) for p in Path(checkpoint_dir).glob("model_*.pt")]
    if not steps:
        raise FileNotFoundError(f"no checkpoints in {checkpoint_dir}")
    return max(steps)
