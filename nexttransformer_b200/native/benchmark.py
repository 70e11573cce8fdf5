"""Timed native-track updates at the fixed global batch (never writes training checkpoints):
``torchrun ... -m nexttransformer_b200.native.benchmark --config configs/native/mor.json
--micro-batch 8 --output bench.json``.

Warm-up updates, then ``--steps`` measured updates with the trainer's own update function; the
report holds the per-step time of the slowest rank, tokens/s, peak memory per rank and the losses.
``--stress-full-path`` forces every token through every routed block (MoR routers and Circle
exits saturated) so that memory is measured at the worst case.
Behaviour: ``nexttransformer/native/benchmark.py:28-135``.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
from dataclasses import asdict
import json
from pathlib import Path
import statistics
import time

import torch
import torch.distributed as dist


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    p.add_argument("--config", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--steps", type=int, default=12)
    p.add_argument("--circle-stage-step", type=int, default=10000)
    p.add_argument("--stress-full-path", action="store_true")
    p.add_argument("--data", choices=("bestfit", "synthetic"), default="synthetic")
    p.add_argument("--global-batch", type=int, default=0)
    a = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(a)
    if a.micro_batch is None or a.warmup < 2 or a.steps < 2:
        p.error("provide --micro-batch; warmup and measured steps must each be >= 2")
    from dataclasses import replace
    from nexttransformer_b200.models.native.config import load_config
    from nexttransformer_b200.models.native.model import build_model, theoretical_training_flops
    from nexttransformer_b200.native.optimizer import build_optimizer, set_schedule
    from nexttransformer_b200.native.train import make_stream, update
    from nexttransformer_b200.runtime.files import atomic_json
    from nexttransformer_b200.runtime.process import initialize, shutdown, synchronize
    mc, tc = load_config(a.config)
    if a.global_batch:
        tc = replace(tc, global_batch_tokens=a.global_batch, total_tokens=a.global_batch * (a.warmup + a.steps))
    rank, world, device = initialize(tc.seed)
    accum = tc.accumulation(mc, world, a.micro_batch)
    stream = make_stream(a, mc, rank, world, tc.seed)
    model = build_model(mc, device, seed=tc.seed)
    optimizer = build_optimizer(model, tc)
    model.train()
    if a.stress_full_path:
        with torch.no_grad():
            if mc.architecture == "mor":
                for r in model.routers:
                    r.weight.zero_()
                    r.bias.fill_(10.)
            elif mc.architecture == "circle":
                model.halter.weight.zero_()
                model.halter.depth_bias.fill_(-10.)
                model.halter.delta_scale.zero_()
    times, losses = [], []
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)
    for step in range(a.warmup + a.steps):
        model.set_circle_step(step + a.circle_stage_step)
        set_schedule(optimizer, step, tc)
        if step == a.warmup and world > 1:
            dist.barrier()
        synchronize(device)
        t0 = time.perf_counter()
        values = update(model, optimizer, stream, mc, tc, accum, a.micro_batch, world, device,
                        step + a.circle_stage_step)
        synchronize(device)
        if values is None:
            raise RuntimeError("non-finite update during the benchmark")
        if step >= a.warmup:
            times.append(time.perf_counter() - t0)
            losses.append(values[0])
    local = {"rank": rank, "step_seconds": times,
             "peak_allocated_bytes": torch.cuda.max_memory_allocated(device) if device.type == "cuda" else 0}
    ranks = [None] * world
    if world > 1:
        dist.all_gather_object(ranks, local)
    else:
        ranks = [local]
    if rank == 0:
        slowest = [max(r["step_seconds"][i] for r in ranks) for i in range(a.steps)]
        report = {"model": asdict(mc), "train": asdict(tc), "world_size": world, "micro_batch": a.micro_batch,
                  "accumulation": accum, "warmup_steps": a.warmup, "measured_steps": a.steps,
                  "step_seconds_max_rank": slowest, "median_step_seconds": statistics.median(slowest),
                  "tokens_per_second": tc.global_batch_tokens * a.steps / sum(slowest),
                  "median_tokens_per_second": tc.global_batch_tokens / statistics.median(slowest),
                  "losses": losses, "ranks": ranks, "train_GFLOPs_per_token": theoretical_training_flops(mc) / 1e9,
                  "torch": torch.__version__, "stress_full_path": a.stress_full_path,
                  "circle_stage_step": a.circle_stage_step}
        atomic_json(a.output, report)
        print(json.dumps({k: report[k] for k in ("micro_batch", "accumulation", "tokens_per_second",
                                                 "median_step_seconds")}), flush=True)
    shutdown()


if __name__ == "__main__":
    main()
