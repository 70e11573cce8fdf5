"""Run tracking: rank-0 JSONL event log (always) mirrored to Weights & Biases when installed.

``start_tracker`` agrees on tracker failure across ranks (all-reduce MAX) before any collective
of the training loop, so every rank fails together (reference ``runtime/tracking.py``).
"""
from contextlib import contextmanager
import json
from pathlib import Path

import torch
import torch.distributed as dist

CORE_KEYS = ("step", "lm_loss", "loss", "grad_norm", "tokens_per_second", "mfu", "val_bpb", "core_metric")


def metric_payload(event, profile="core"):
    """Flat numeric metrics of an event for the tracker."""
    keys = CORE_KEYS if profile == "core" else event.keys()
    return {k: v for k, v in event.items() if k in keys and isinstance(v, (int, float)) and not isinstance(v, bool)}


class RunTracker:
    def __init__(self, output, rank, mode="disabled", config=None, run_id=None):
        self.output, self.rank, self.mode = Path(output), rank, mode
        self.run = None
        if rank == 0 and mode != "disabled":
            try:
                import wandb
                self.run = wandb.init(project="nexttransformer_b200", mode=mode, config=config or {}, id=run_id,
                                      resume="allow", dir=str(self.output))
            except ImportError:
                self.run = None

    def log(self, event):
        if self.rank != 0:
            return
        self.output.mkdir(parents=True, exist_ok=True)
        with (self.output / "metrics.jsonl").open("a") as f:
            f.write(json.dumps(event, ensure_ascii=False) + "\n")
        if self.run is not None:
            self.run.log(metric_payload(event), step=event.get("step"))

    def close(self):
        if self.run is not None:
            self.run.finish()


@contextmanager
def start_tracker(output, rank, mode="disabled", config=None, device=None):
    failed = 0
    tracker = None
    try:
        tracker = RunTracker(output, rank, mode, config)
    except Exception:
        failed = 1
    if dist.is_initialized():
        flag = torch.tensor([failed], device=device or "cpu")
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        failed = int(flag.item())
    if failed:
        raise RuntimeError("run tracker failed to start on at least one rank")
    try:
        yield tracker
    finally:
        tracker.close()
