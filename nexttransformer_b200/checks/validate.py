"""Bounded per-method architecture checks (no optimizer update).

    python -m nexttransformer_b200.checks.validate --output val.json [--mode smoke|target] [--device cpu]

For each method (ranks take disjoint methods under torchrun): build it (debug size in ``smoke``
mode, the registered configuration in ``target`` mode), perturb the zero-initialised output
projections so every path carries signal, run forward + backward on random tokens, require a finite
loss and a finite gradient for every trainable parameter, then check causality: changing the second
half of the tokens must leave the first half's logits unchanged.  Failures are recorded per method.
Behaviour: ``nexttransformer/checks/validate.py:40-133``.
"""
import argparse
from datetime import datetime, timezone
import gc
import json
import os
from pathlib import Path
import time
import traceback

import torch
import torch.distributed as dist


def activate(model):
    with torch.no_grad():
        for blk in model.transformer.h:
            blk.attn.c_proj.weight.normal_(std=.02)
            blk.mlp.c_proj.weight.normal_(std=.02)


def check_one(method, args, device):
    from nexttransformer_b200.models.config import candidate_config, debug_config
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.optim.muon_adamw import grad_of
    from nexttransformer_b200.protocol.spec import config_file, load_config
    if args.config_dir:
        c = load_config(config_file(args.config_dir, method))
    else:
        c = candidate_config(method) if args.mode == "target" else debug_config(method)
    model = build_model(c, device, seed=42)
    activate(model)
    model.set_step(0 if args.stage == "burnin" else c.burnin_steps + 1)
    T = args.sequence_length or (64 if args.mode == "target" else c.sequence_len)
    if T > c.sequence_len:
        raise ValueError("test length exceeds the model context")
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randint(c.vocab_size, (args.micro_batch, T), generator=g).to(device)
    y = torch.randint(c.vocab_size, x.shape, generator=g).to(device)
    t0 = time.monotonic()
    loss = model(x, y)
    loss.backward()
    if not torch.isfinite(loss):
        raise RuntimeError("non-finite loss")
    missing = []
    for name, q in model.named_parameters():
        gr = grad_of(q)
        if q.requires_grad and gr is None:
            missing.append(name)
        if gr is not None and not torch.isfinite(gr).all():
            raise RuntimeError("non-finite gradient: " + name)
    if missing:
        raise RuntimeError("missing gradients: " + ", ".join(missing))
    model.zero_grad(set_to_none=True)
    model.eval()
    with torch.no_grad():
        z = x.clone()
        z[:, T // 2:] = (z[:, T // 2:] + 7) % c.vocab_size
        err = float((model(x)[:, :T // 2] - model(z)[:, :T // 2]).abs().max())
    if err > 3e-3:
        raise RuntimeError(f"causal prefix changed: {err}")
    return dict(method=method, status="passed", mode=args.mode, model_hash=c.fingerprint, test_shape=list(x.shape),
                width=c.width, physical_layers=c.n_layer, parameters=sum(q.numel() for q in model.parameters()),
                loss=float(loss.detach()), causal_max_abs=err, elapsed_seconds=time.monotonic() - t0,
                stage=args.stage)


def main(argv=None):
    from nexttransformer_b200.models.registry import METHODS
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--mode", choices=("smoke", "target"), default="smoke")
    p.add_argument("--methods", nargs="+", choices=METHODS, default=list(METHODS))
    p.add_argument("--device", choices=("cpu", "cuda"), default="cuda")
    p.add_argument("--sequence-length", type=int)
    p.add_argument("--micro-batch", type=int, default=1)
    p.add_argument("--config-dir")
    p.add_argument("--stage", choices=("burnin", "joint"), default="joint")
    p.add_argument("--output", required=True)
    a = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    device = torch.device("cuda", local) if a.device == "cuda" else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("gloo")
    results = []
    for method in a.methods[rank::world]:
        try:
            res = check_one(method, a, device)
        except Exception as e:     # recorded, never hidden: the exit code reports it
            res = dict(method=method, status="failed", error=str(e), traceback=traceback.format_exc())
        gc.collect()
        results.append(res)
        print(json.dumps(dict(rank=rank, **res)), flush=True)
    out = Path(a.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    shard = out.with_name(f"{out.stem}.rank{rank}{out.suffix}")
    shard.write_text(json.dumps(results, indent=2) + "\n")
    if world > 1:
        dist.barrier()
    if rank == 0:
        merged = []
        for r in range(world):
            merged += json.loads(out.with_name(f"{out.stem}.rank{r}{out.suffix}").read_text())
        out.write_text(json.dumps(dict(created_at=datetime.now(timezone.utc).isoformat(), torch=torch.__version__,
                                       device=str(device), world_size=world, mode=a.mode, results=merged),
                                  indent=2) + "\n")
    if world > 1:
        dist.destroy_process_group()
    if any(r["status"] != "passed" for r in results):
        raise SystemExit(1)
    return results


if __name__ == "__main__":
    main()
