"""Checkpoints for nodes that share no filesystem (``nexttransformer/scaling/checkpoint.py`` of the
reference).

Every node writes a self-contained copy under ``checkpoint_%08d/node_%03d/``: the model, both
configurations and the run state from the node's first rank, one optimizer / RNG / data-cursor /
routing-RNG shard per rank, and last a ``complete.json`` that lists every rank's files with size and
sha256 and the rank layout.  A restart takes the newest step complete on every node (the sets of
complete steps are exchanged with all_gather_object), sets this node's newer checkpoints aside
(never deletes them), and loads only after every rank agrees that its files pass the checksums
and the rank layout is unchanged.
"""
from dataclasses import asdict
import json
import os
from pathlib import Path
import shutil
import socket
import time

import torch
import torch.distributed as dist

from nexttransformer_b200.runtime.checkpoint import load_optimizer_state
from nexttransformer_b200.runtime.files import atomic_json, sha256
from nexttransformer_b200.runtime.process import restore_rng, rng_state


def _world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def topology():
    """(node, local_rank, local_world): torchrun places each node's ranks in one contiguous block."""
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    return rank // local_world, int(os.environ.get("LOCAL_RANK", "0")), local_world


def gather(value):
    """Every rank's `value` (picklable), in rank order."""
    if _world()[1] == 1:
        return [value]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, value)
    return out


def agree(ok, device):
    """True only when every rank reports ok (one MIN all-reduce)."""
    if _world()[1] == 1:
        return bool(ok)
    flag = torch.tensor([1 if ok else 0], device=device, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def node_directory(output, step, node):
    return Path(output) / f"checkpoint_{step:08d}" / f"node_{node:03d}"


def complete_steps(output, node):
    steps = []
    for marker in Path(output).glob(f"checkpoint_[0-9]*/node_{node:03d}/complete.json"):
        steps.append(int(marker.parent.parent.name[len("checkpoint_"):]))
    return sorted(steps)


def common_step(output):
    """The newest step complete on every node (None when there is none)."""
    node, _, _ = topology()
    shared = None
    for steps in gather(complete_steps(output, node)):
        shared = set(steps) if shared is None else shared & set(steps)
    return max(shared) if shared else None


def set_aside_after(output, step, node=None):
    """Move this node's checkpoints newer than `step` (complete or partial) to ``abandoned/``.
    Only the node's first rank moves; every rank may call."""
    if node is None:
        node, local_rank, _ = topology()
        if local_rank:
            return []
    step = -1 if step is None else step
    archive = Path(output) / "abandoned" / str(time.time_ns())
    moved = []
    for path in sorted(Path(output).glob(f"checkpoint_[0-9]*/node_{node:03d}")):
        if int(path.parent.name[len("checkpoint_"):]) <= step:
            continue
        target = archive / path.parent.name / path.name
        target.parent.mkdir(parents=True, exist_ok=True)
        path.rename(target)
        moved.append(path.parent.name)
        try:
            path.parent.rmdir()
        except OSError:
            pass
    return moved


def prune(output, node, keep):
    """Delete this node's oldest complete rolling checkpoints beyond `keep`; milestones stay."""
    if keep < 2:
        raise ValueError("keep at least two rolling checkpoints so a common restart point survives")
    rolling = []
    for step in complete_steps(output, node):
        d = node_directory(output, step, node)
        if not json.loads((d / "complete.json").read_text())["milestone"]:
            rolling.append(d)
    for d in rolling[:-keep]:
        shutil.rmtree(d)
        try:
            d.parent.rmdir()
        except OSError:
            pass


def _routing_state(model):
    return model.routing_rng_state() if hasattr(model, "routing_rng_state") else None


def save_checkpoint(output, model, optimizer, stream, mc, tc, state, milestone=False):
    node, local_rank, local_world = topology()
    rank, world = _world()
    directory = node_directory(output, state["step"], node)
    if local_rank == 0:
        directory.mkdir(parents=True, exist_ok=False)
    if world > 1:
        dist.barrier()
    files = {}

    def put(name, payload):
        tmp = directory / (name + ".tmp")
        torch.save(payload, tmp)
        tmp.replace(directory / name)
        files[name] = {"bytes": (directory / name).stat().st_size, "sha256": sha256(directory / name)}

    put(f"rank_{rank:04d}.pt", {"optimizer": optimizer.state_dict(), "rng": rng_state(),
                                "data": stream.state_dict(), "routing_rng": _routing_state(model)})
    if local_rank == 0:
        put("model.pt", {"model": model.state_dict(), "model_config": mc.serialized(), "train_config": asdict(tc),
                         "state": state, "world_size": world, "local_world_size": local_world})
    nodes = {}
    for entry in gather({"node": node, "host": socket.gethostname(), "files": files}):
        slot = nodes.setdefault(f"{entry['node']:03d}", {"host": entry["host"], "files": {}})
        slot["files"].update(entry["files"])
    if local_rank == 0:
        atomic_json(directory / "complete.json", {"step": state["step"], "world_size": world,
                                                  "local_world_size": local_world, "milestone": milestone,
                                                  "nodes": dict(sorted(nodes.items()))})
    if world > 1:
        dist.barrier()
    return directory


def load_checkpoint(output, step, model, optimizer, stream, device):
    node, local_rank, local_world = topology()
    rank, world = _world()
    directory = node_directory(output, step, node)
    try:
        record = json.loads((directory / "complete.json").read_text())
        files = record["nodes"][f"{node:03d}"]["files"]
        needed = [f"rank_{rank:04d}.pt"] + (["model.pt"] if local_rank == 0 else [])
        ok = (record["world_size"], record["local_world_size"]) == (world, local_world) and all(
            (directory / n).stat().st_size == files[n]["bytes"] and sha256(directory / n) == files[n]["sha256"]
            for n in needed)
    except (OSError, KeyError, ValueError):
        ok = False
    if not agree(ok, device):
        raise ValueError(f"checkpoint {step} is missing, has another rank layout or fails a checksum on some rank")
    saved = torch.load(directory / "model.pt", map_location="cpu", weights_only=False)
    model.load_state_dict(saved["model"], strict=True)
    local = torch.load(directory / f"rank_{rank:04d}.pt", map_location="cpu", weights_only=False)
    load_optimizer_state(optimizer, local["optimizer"])
    stream.load_state_dict(local["data"])
    restore_rng(local["rng"])
    if local["routing_rng"] is not None and hasattr(model, "restore_routing_rng"):
        model.restore_routing_rng(local["routing_rng"])
    return saved
