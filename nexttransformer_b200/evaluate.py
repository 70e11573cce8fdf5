"""Evaluate a checkpoint: ``python -m nexttransformer_b200.evaluate --checkpoint DIR [--bpb] [--core BUNDLE]``.

BPB runs on the validation split of the parquet data (with a tokenizer) or on the held-out
synthetic stream; CORE runs on a local task bundle (JSON lines per task plus a task list), with
examples sharded over ranks.  Results are written atomically by rank 0.
"""
import argparse
import json
from pathlib import Path

import torch


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--checkpoint", type=Path, required=True)
    p.add_argument("--output", type=Path)
    p.add_argument("--tokens", type=int, default=1 << 20)
    p.add_argument("--micro-batch", type=int, default=8)
    p.add_argument("--data-dir", type=Path)
    p.add_argument("--tokenizer", type=Path)
    p.add_argument("--core", type=Path, help="directory with tasks.json and <label>.jsonl files")
    p.add_argument("--core-max-per-task", type=int, default=-1)
    from nexttransformer_b200.evaluation.context import add_core_max_tokens
    add_core_max_tokens(p)
    p.add_argument("--expected-attention", help="refuse to run unless this attention path is active")
    a = p.parse_args(argv)
    from nexttransformer_b200.evaluation.bpb import evaluate_bpb, evaluate_stream_loss
    from nexttransformer_b200.models import load_model
    from nexttransformer_b200.runtime.files import atomic_json
    from nexttransformer_b200.runtime.process import initialize, shutdown
    rank, world, dev = initialize(42)
    model, saved = load_model(a.checkpoint, dev)
    if a.expected_attention:
        active = "sm100_flash" if dev.type == "cuda" else "sdpa"
        if active != a.expected_attention:
            raise SystemExit(f"attention path is {active}, expected {a.expected_attention}")
    cfg = model.config
    result = {"step": saved["state"]["step"]}
    if a.data_dir and a.tokenizer:
        from nexttransformer_b200.runtime.data import BestFitStream
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tok = BPETokenizer.from_directory(a.tokenizer)
        stream = BestFitStream(a.data_dir, tok, "val", rank, world, cfg.sequence_len)
        steps = max(1, a.tokens // (world * a.micro_batch * cfg.sequence_len))
        result["val_bpb"] = evaluate_bpb(model, stream.batches(a.micro_batch, dev), steps, tok.token_bytes().to(dev))
    else:
        result.update(evaluate_stream_loss(model, cfg, a.tokens, a.micro_batch, rank, world, dev))
    if a.core:
        from nexttransformer_b200.evaluation.core import evaluate_core
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tok = BPETokenizer.from_directory(a.tokenizer)
        tasks = json.loads((a.core / "tasks.json").read_text())
        for t in tasks:
            t["data"] = [json.loads(l) for l in (a.core / f"{t['label']}.jsonl").read_text().splitlines() if l]
        from nexttransformer_b200.evaluation.context import (LengthProbe, check_full_context, core_context,
                                                             inference_view)
        if a.core_max_per_task <= 0:
            check_full_context(cfg, a.core_max_tokens)
        model.eval()
        probe = LengthProbe(inference_view(model, a.core_max_tokens))
        result["core"] = evaluate_core(probe, tok, tasks, dev, rank, world, a.core_max_per_task, a.core_max_tokens)
        longest = torch.tensor(probe.longest, device=dev)
        if world > 1:
            torch.distributed.all_reduce(longest, op=torch.distributed.ReduceOp.MAX)
        result["core"]["coreContext"] = core_context(cfg.sequence_len, a.core_max_tokens, int(longest.item()))
    if rank == 0:
        print(json.dumps(result))
        if a.output:
            atomic_json(a.output, result)
    shutdown()
    return result


if __name__ == "__main__":
    main()
