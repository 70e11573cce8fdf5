"""Scheduled evaluation of a training run: validation bits per byte, CORE and the final evaluation.

``RunEvaluator`` holds what a trainer needs to evaluate its model between updates:

* ``validation(tokens, split)``: bits per byte on a split of the prepared dataset (BOS best-fit
  rows, the same per-rank stream layout as training, partial sums all-reduced) when the run trains
  on real data, else the mean token loss of a held-out synthetic stream (research runs without a
  dataset);
* ``core(final)``: CORE-22 centred accuracy through the inference view of the model (full prompts
  beyond the training context up to ``core_max_tokens``), with the longest prompt seen recorded
  as ``coreContext``;
* ``final()``: the train and validation splits at the final-evaluation budget.

Behaviour follows the reference trainer's ``validation`` / ``core`` / final evaluation
(``nexttransformer/train.py:420-462,557-567``).
"""
import json
import time
from pathlib import Path

import torch
import torch.distributed as dist


def load_core_bundle(path):
    """CORE tasks of a bundle directory: ``tasks.json`` plus one ``<label>.jsonl`` per task."""
    path = Path(path)
    tasks = json.loads((path / "tasks.json").read_text())
    for task in tasks:
        task["data"] = [json.loads(line) for line in (path / f"{task['label']}.jsonl").read_text().splitlines() if line]
    return tasks


class RunEvaluator:
    def __init__(self, model, config, *, rank, world, device, micro, data="synthetic", data_dir=None,
                 tokenizer=None, core_tasks=None, core_max_tokens=None, core_max_per_task=-1, seed=0,
                 stream_rank=None, stream_world=None):
        self.model, self.config = model, config
        self.rank, self.world, self.device, self.micro = rank, world, device, micro
        self.data, self.data_dir, self.tokenizer = data, data_dir, tokenizer
        self.tasks, self.core_max_tokens, self.core_max_per_task = core_tasks, core_max_tokens, core_max_per_task
        self.seed = seed
        self.stream_rank = rank if stream_rank is None else stream_rank
        self.stream_world = world if stream_world is None else stream_world
        self.seconds = 0.0

    # ------------------------------------------------------------------ validation
    def validation(self, tokens, split="val"):
        t0 = time.time()
        if self.data == "synthetic" or self.tokenizer is None:
            from nexttransformer_b200.evaluation.bpb import evaluate_stream_loss
            result = evaluate_stream_loss(self.model, self.config, tokens, self.micro, self.rank, self.world,
                                          self.device, self.seed + (0 if split == "val" else 1))
            result = {"split": split, **result}
        else:
            from nexttransformer_b200.evaluation.bpb import evaluate_bpb
            from nexttransformer_b200.runtime.data import BestFitStream
            T = self.config.sequence_len
            stream = BestFitStream(self.data_dir, self.tokenizer, split, self.stream_rank, self.stream_world, T)
            steps = max(1, tokens // (self.world * self.micro * T))
            bpb = evaluate_bpb(self.model, stream.batches(self.micro, self.device), steps,
                               self.tokenizer.token_bytes().to(self.device))
            result = {"split": split, "bpb": bpb, "input_tokens": steps * self.world * self.micro * T}
        result["seconds"] = time.time() - t0
        self.seconds += result["seconds"]
        return result

    def final(self, tokens):
        return {split: self.validation(tokens, split) for split in ("train", "val")}

    # ------------------------------------------------------------------ CORE
    @property
    def has_core(self):
        return self.tasks is not None and self.tokenizer is not None

    def core(self, final=False):
        from nexttransformer_b200.evaluation.context import LengthProbe, core_context, inference_view
        from nexttransformer_b200.evaluation.core import evaluate_core
        t0 = time.time()
        model = self.model
        was = model.training
        model.eval()             # before the view: the shallow copy keeps the mode it was made in
        backend = None
        if hasattr(model, "set_sparse_backend"):
            backend = next((b.attn.backend for b in model.transformer.h if hasattr(b.attn, "backend")), None)
            if backend is not None:
                model.set_sparse_backend("reference")
        try:
            probe = LengthProbe(inference_view(model, self.core_max_tokens))
            with torch.no_grad():
                result = evaluate_core(probe, self.tokenizer, self.tasks, self.device, self.rank, self.world,
                                       -1 if final else self.core_max_per_task, self.core_max_tokens)
        finally:
            if backend is not None:
                model.set_sparse_backend(backend)
            model.train(was)
        longest = torch.tensor(probe.longest, device=self.device)
        if dist.is_initialized() and self.world > 1:
            dist.all_reduce(longest, op=dist.ReduceOp.MAX)
        result["coreContext"] = core_context(self.config.sequence_len, self.core_max_tokens, int(longest.item()))
        result["seconds"] = time.time() - t0
        self.seconds += result["seconds"]
        return result
