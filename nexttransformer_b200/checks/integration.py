"""Bounded checks on the real resources: the data cursor, the BPB evaluator and a CORE smoke run
(``nexttransformer/checks/integration.py`` of the reference).

    python -m nexttransformer_b200.checks.integration --data-dir DATA --resources RES --output out.json \
        [--core BUNDLE] [--device cuda]

* data: the BOS best-fit stream packs the same rows whatever the micro-batch size (4 rows at once ==
  2 + 2), and a stream restored from its state continues with the same rows;
* BPB: ``evaluation.bpb.evaluate_bpb`` equals a direct fp64 recomputation (per-token losses of the
  same model, target byte lengths from ``token_bytes.pt``) on the validation split;
* CORE: tiny models of a few registered methods score a bounded sample of every task.
Models are tiny-width debug configurations at the tokenizer's vocabulary: the check covers
interfaces, never model quality.  The output JSON carries the resource fingerprints and the flags.
"""
import argparse
from dataclasses import replace
import hashlib
import json
import math
import os
from pathlib import Path

import torch
import torch.distributed as dist


def checksum(x, y):
    return hashlib.sha256(x.cpu().numpy().tobytes() + y.cpu().numpy().tobytes()).hexdigest()


def _tiny(method, vocab, sequence_len, device):
    from nexttransformer_b200.models import build_model
    from nexttransformer_b200.models.config import debug_config
    cfg = replace(debug_config(method), vocab_size=vocab, sequence_len=sequence_len)
    return build_model(cfg, device, seed=7).eval()


@torch.no_grad()
def direct_bpb(model, batches, steps, token_bytes):
    nats, nbytes = 0.0, 0
    for _ in range(steps):
        x, y = next(batches)
        loss = model(x, y, loss_reduction="none").reshape(-1).double()
        b = token_bytes[y.reshape(-1).clamp_min(0)].long() * (y.reshape(-1) >= 0)
        nats += float((loss * (b > 0)).sum())
        nbytes += int(b.sum())
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([nats, float(nbytes)], dtype=torch.float64, device=token_bytes.device)
        dist.all_reduce(t)
        nats, nbytes = float(t[0]), int(t[1])
    return nats / (math.log(2) * max(nbytes, 1))


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--data-dir", type=Path, required=True)
    p.add_argument("--resources", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--device", default="cuda", choices=("cpu", "cuda"))
    p.add_argument("--sequence-len", type=int, default=2048)
    p.add_argument("--bpb-steps", type=int, default=2)
    p.add_argument("--core", type=Path, help="CORE bundle (tasks.json + <label>.jsonl)")
    p.add_argument("--core-methods", nargs="*", default=["dense", "huginn", "qsa", "kda"])
    p.add_argument("--core-max-per-task", type=int, default=32,
                   help="the smoke pool must exceed the largest few-shot count (10)")
    a = p.parse_args(argv)
    from nexttransformer_b200.evaluation.bpb import evaluate_bpb
    from nexttransformer_b200.protocol.spec import Protocol
    from nexttransformer_b200.runtime.data import BestFitStream
    from nexttransformer_b200.runtime.resources import tokenizer_fingerprint, verify_resources
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    if a.core and a.core_max_per_task <= 10:
        raise ValueError("the CORE smoke pool must hold more than 10 examples for few-shot sampling")
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if a.device == "cuda":
        torch.cuda.set_device(local)
    device = torch.device("cuda", local) if a.device == "cuda" else torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl" if a.device == "cuda" else "gloo")
    _, manifest = verify_resources(a.resources, a.data_dir)
    tok = BPETokenizer.from_directory(a.resources / "tokenizer")
    vocab = tok.get_vocab_size()
    T = a.sequence_len
    s1 = BestFitStream(a.data_dir, tok, "train", rank, world, T)
    s2 = BestFitStream(a.data_dir, tok, "train", rank, world, T)
    ax, ay = s1.batch(4, device)
    bx1, by1 = s2.batch(2, device)
    state = s2.state_dict()
    bx2, by2 = s2.batch(2, device)
    if not (torch.equal(ax, torch.cat((bx1, bx2))) and torch.equal(ay, torch.cat((by1, by2)))):
        raise RuntimeError("packing changed with the micro-batch size")
    s2.load_state_dict(state)
    rx, ry = s2.batch(2, device)
    if not (torch.equal(rx, bx2) and torch.equal(ry, by2)):
        raise RuntimeError("a restored stream continued with other rows")
    model = _tiny("dense", vocab, T, device)
    token_bytes = torch.load(a.resources / "tokenizer" / "token_bytes.pt", map_location=device, weights_only=True)
    got = evaluate_bpb(model, BestFitStream(a.data_dir, tok, "val", rank, world, T).batches(2, device), a.bpb_steps,
                       token_bytes)
    want = direct_bpb(model, BestFitStream(a.data_dir, tok, "val", rank, world, T).batches(2, device), a.bpb_steps,
                      token_bytes)
    if not math.isclose(got, want, rel_tol=1e-9):
        raise RuntimeError(f"BPB evaluator {got} differs from the direct computation {want}")
    del model
    core = []
    out = dict(status="running", protocol_hash=Protocol().fingerprint, data_manifest_sha256=manifest,
               tokenizer_sha256=tokenizer_fingerprint(a.resources), data_rows_sha256=checksum(ax, ay),
               microbatch_data_equal=True, resume_rows_equal=True, bpb_exact=True, bpb_smoke=got, core_smoke=core,
               world_size=world, formal_evaluation=False, torch=torch.__version__)

    def save(status):
        if rank == 0:
            out["status"] = status
            a.output.parent.mkdir(parents=True, exist_ok=True)
            a.output.write_text(json.dumps(out, indent=2) + "\n")
    save("running")
    if a.core:
        from nexttransformer_b200.evaluation.core import evaluate_core
        tasks = json.loads((a.core / "tasks.json").read_text())
        for t in tasks:
            t["data"] = [json.loads(l) for l in (a.core / f"{t['label']}.jsonl").read_text().splitlines() if l]
        for method in a.core_methods:
            model = _tiny(method, vocab, T, device)
            with torch.no_grad():
                result = evaluate_core(model, tok, tasks, device, rank, world, a.core_max_per_task, T)
            core.append(dict(method=method, status="passed", full_core=False, core_metric=result["core_metric"]))
            save("running")
            del model
    save("passed")
    if rank == 0:
        print(json.dumps(dict(status="passed", bpb_exact=True, core_methods=len(core))), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
