"""One bounded multi-rank optimizer update per method (never a training run).

    torchrun --nproc-per-node 8 -m nexttransformer_b200.checks.distributed --output dist.json [--methods ...]

Each method is built at debug width with real ``sequence_len`` rows; every rank feeds stateless
token rows (``(pos mod (T+1) + row*17 + 42) mod vocab``, invariant to micro-batch splitting) so the
global batch is the protocol's (or, with ``--smoke``, any batch the ranks divide).  After one update
the check requires finite gradients for every trainable parameter, a real parameter change and a
parameter digest that is equal on every rank.  Synthetic data is labelled as such.
Behaviour: ``nexttransformer/checks/distributed.py:38-108``.
"""
import argparse
from datetime import datetime, timezone
import gc
import json
from pathlib import Path
import time

import torch
import torch.distributed as dist


def main(argv=None):
    from nexttransformer_b200.models.registry import METHODS
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--methods", nargs="+", choices=METHODS, default=list(METHODS))
    p.add_argument("--micro-batch", type=int, default=64)
    p.add_argument("--full-dimensions", action="store_true")
    p.add_argument("--config-dir", type=Path, default=Path("configs"))
    p.add_argument("--sequence-len", type=int, default=0, help="row length (0: the protocol's)")
    p.add_argument("--global-batch", type=int, default=0, help="tokens per update (0: the protocol's)")
    p.add_argument("--smoke", action="store_true")
    p.add_argument("--output", type=Path, required=True)
    a = p.parse_args(argv)
    from nexttransformer_b200.checks.common import parameter_digest, source_hash
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.optim.groups import protocol_groups, set_schedule
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW, grad_of
    from nexttransformer_b200.protocol.spec import Protocol, config_file, load_config
    from nexttransformer_b200.runtime.process import initialize, shutdown
    src = source_hash()
    proto = Protocol()
    rank, world, device = initialize(42)
    T = a.sequence_len or proto.sequence_len
    gb = a.global_batch or proto.global_batch_tokens
    per = world * a.micro_batch * T
    if gb % per:
        raise ValueError("micro-batch x ranks x sequence must divide the global batch")
    accum = gb // per
    results = []
    for method in a.methods:
        c = load_config(config_file(a.config_dir, method)) if a.full_dimensions else debug_config(method,
                                                                                                   sequence_len=T)
        model = build_model(c, device, seed=42)
        step = c.burnin_steps + 1
        model.set_training_stage(step)
        model.set_step(min(step, proto.steps))
        shadows = {}
        if device.type == "cuda":
            shadows = {q: s for q, s in model.fused_state().casts}
        opt = MuonAdamW(protocol_groups(model), shadows=shadows)
        set_schedule(opt, step, proto.train_config())
        before = parameter_digest(model)
        if world > 1:
            dist.barrier()
        t0 = time.monotonic()
        rows = gb // T // world
        total = torch.zeros((), device=device)
        for m in range(accum):
            first = rank * rows + m * a.micro_batch
            model.set_row_offset(first)
            pos = torch.arange(a.micro_batch * (T + 1), device=device).reshape(a.micro_batch, -1)
            ids = torch.arange(first, first + a.micro_batch, device=device)[:, None]
            tok = (pos.remainder(T + 1) + ids * 17 + 42).remainder(c.vocab_size)
            x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
            loss = model(x, y) / accum
            loss.backward()
            total += loss.detach()
        for name, q in model.named_parameters():
            g = grad_of(q)
            if q.requires_grad and (g is None or not torch.isfinite(g).all()):
                raise RuntimeError("missing or non-finite gradient: " + name)
        opt.step()
        if device.type == "cuda":
            torch.cuda.synchronize()
        seconds = time.monotonic() - t0
        after = parameter_digest(model)
        digests = [None] * world
        if world > 1:
            dist.all_gather_object(digests, after)
            dist.all_reduce(total)
        else:
            digests = [after]
        if len(set(digests)) != 1 or before == after:
            raise RuntimeError(f"{method}: the update was not real or not synchronized")
        res = dict(method=method, status="passed", model_hash=c.fingerprint, full_dimensions=a.full_dimensions,
                   input_shape=[a.micro_batch, T], global_tokens=gb, world_size=world, accumulation=accum,
                   optimizer_updates=1, loss=float(total / world), seconds=seconds, all_rank_parameters_equal=True,
                   peak_allocated_bytes=torch.cuda.max_memory_allocated() if device.type == "cuda" else None,
                   synthetic_data=True, smoke=a.smoke)
        results.append(res)
        if rank == 0:
            if source_hash() != src:
                raise RuntimeError("sources changed during the check")
            print(json.dumps(res), flush=True)
            a.output.parent.mkdir(parents=True, exist_ok=True)
            a.output.write_text(json.dumps(dict(created_at=datetime.now(timezone.utc).isoformat(), source_hash=src,
                                                protocol_hash=proto.fingerprint, torch=torch.__version__,
                                                device=str(device), results=results), indent=2) + "\n")
        del opt, model
        gc.collect()
        if device.type == "cuda":
            torch.cuda.empty_cache()
        if world > 1:
            dist.barrier()
    shutdown()
    return results


if __name__ == "__main__":
    main()
