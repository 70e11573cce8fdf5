"""Counted evaluation of the native-track models: BPB and CORE with route accounting.

Every forward of the native models (``models/native/model.py``) leaves ``last_stats``: input
tokens, forward FLOPs of the executed work, the summed active depth and the tokens still active at
each routing step.  An evaluation here wraps the model so those counters are summed over every
evaluation forward and reduced over ranks, and reports them beside the score: the mean active
depth, the per-step active ratios and the mean recursion count (ring steps, exit ratios and the cap
ratio for Circle).  Behaviour follows the reference's ``nexttransformer/evaluation/native.py:14-64``
and ``evaluation/metrics.py:8-29``; BPB and CORE themselves are this package's
``evaluation/bpb.py`` and ``evaluation/core.py``.
"""
import time

import torch
import torch.distributed as dist


class RouteCounter:
    """Sums of the native models' forward statistics; ``result`` reduces them over ranks."""

    def __init__(self, steps, circle=False):
        self.steps, self.circle = steps, circle
        self.tokens = self.flops = self.depth = 0.0
        self.active = [0.0] * steps

    def add(self, stats):
        self.tokens += stats["input_tokens"]
        self.flops += stats["forward_flops"]
        self.depth += stats["active_depth_sum"]
        for i, n in enumerate(stats["active_tokens"]):
            self.active[i] += n

    def result(self, device):
        v = torch.tensor([self.tokens, self.flops, self.depth, *self.active], dtype=torch.float64, device=device)
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(v)
        tokens, flops, depth, *active = v.tolist()
        n = max(tokens, 1.0)
        out = {"input_tokens": int(tokens), "forward_flops_estimate": flops, "mean_active_depth": depth / n,
               "active_ratios": [a / n for a in active]}
        if self.circle:
            out["mean_ring_steps"] = sum(active) / n
            reached = active + [0.0]
            out["exit_ratios"] = [(reached[i] - reached[i + 1]) / n for i in range(self.steps)]
            out["cap_ratio"] = active[-1] / n
        else:
            out["mean_recursions"] = sum(active) / n
        return out


class Counted(torch.nn.Module):
    """The model, with each forward's ``last_stats`` added to a counter."""

    def __init__(self, model, counter):
        super().__init__()
        self.model, self.counter = model, counter
        self.config = model.config

    def forward(self, *args, **kwargs):
        out = self.model(*args, **kwargs)
        self.counter.add(self.model.last_stats)
        return out


def _counter(model):
    c = model.config
    return RouteCounter(c.routing_steps, c.architecture == "circle")


def _sync(device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@torch.no_grad()
def evaluate_native_bpb(model, tokenizer, data_dir, tokens, batch, rank, world, device, split="val"):
    """BPB of ``split`` over exactly ``tokens`` input tokens of the BOS best-fit stream (rank-strided
    rows), with the route accounting of those forwards."""
    from nexttransformer_b200.evaluation.bpb import evaluate_bpb
    from nexttransformer_b200.runtime.data import BestFitStream
    T = model.config.sequence_len
    per_step = batch * world * T
    if tokens % per_step:
        raise ValueError("the BPB token budget must be a multiple of the distributed evaluation batch")
    stream = BestFitStream(data_dir, tokenizer, split, rank, world, T)
    counter = _counter(model)
    was = model.training
    model.eval()
    _sync(device)
    t0 = time.perf_counter()
    try:
        value = evaluate_bpb(Counted(model, counter), stream.batches(batch, device), tokens // per_step,
                             tokenizer.token_bytes().to(device))
        result = counter.result(device)
        _sync(device)
        if result["input_tokens"] != tokens:
            raise RuntimeError("BPB evaluation read a different number of tokens than its budget")
        return {**result, f"{split}_bpb": value, "seconds": time.perf_counter() - t0, "split": split,
                "protocol": "nanochat_bos_bestfit"}
    finally:
        model.train(was)


@torch.no_grad()
def evaluate_native_core(model, tokenizer, tasks, device, rank=0, world=1, max_per_task=-1, max_len=None):
    """CORE-22 through the counted model; ``full_core`` is True when every example was scored."""
    from nexttransformer_b200.evaluation.core import evaluate_core
    counter = _counter(model)
    was = model.training
    model.eval()
    _sync(device)
    t0 = time.perf_counter()
    try:
        result = evaluate_core(Counted(model, counter), tokenizer, tasks, device, rank, world, max_per_task, max_len)
        result.update(counter.result(device))
        _sync(device)
        return {**result, "seconds": time.perf_counter() - t0, "full_core": max_per_task <= 0,
                "entries": len(tasks)}
    finally:
        model.train(was)
