#!/usr/bin/env python
"""Headline benchmark: train tokens/s (all GPUs, max-over-ranks device time) of the dense GQA
decoder of the benchmark configuration, at a global batch of 524,288 tokens per update.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--method M]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1)

Without ``--method`` (or with ``dense``) the headline configuration below runs.  ``--method``
selects another benchmark configuration of the survey on the generic model path
(``models.build_model``): ``gdn_hybrid_swa`` / ``kda_hybrid`` (depth 24, width 1536, 12 heads of
128, chunk 64, sequence 4096, 524,288 tokens per update), ``nsa`` / ``moba`` (depth 24, width
1536, 16 query heads of 128 / 1 KV head, sequence 8192) and ``moe`` (depth 16, width 2048, 16 / 4 heads,
64 experts of FFN 1024, top-8 + 1 shared, sequence 4096, 1,048,576 tokens per update).

Model: depth 20, width 1280, 10 query heads / 5 KV heads of dim 128, RoPE, RMSNorm, ReLU^2 MLP
4x, vocab 65536, sequence 2048, on the shared shell (value embeddings, smear, backout, soft-cap
15) - the reference's own shell class with these dimensions, so both arms train the same network.
Optimizer: Muon + AdamW (the shell recipe), one update per step.  Data: iid uniform synthetic
tokens, random-init weights.  Strong scaling: the global batch is fixed and every GPU runs
global / N tokens per update (gradient accumulation below 8 GPUs).

Two numbers are reported: ``value`` times the update on device-resident inputs (CUDA events,
barrier + synchronize on both sides, max over ranks); ``e2e.value`` times the public
``Trainer.step`` call, which copies every micro-batch host->device from pinned memory and
reads the loss back.  The working set (activations of 32 x 2048 tokens) is far larger than
L2, so no explicit flush is needed between timed steps.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE_TOKS = None  # the reference publishes no number for this configuration
MODEL = dict(sequence_len=2048, vocab_size=65536, n_layer=20, n_head=10, n_kv_head=5, n_embd=1280,
             window_pattern="L")
GLOBAL_BATCH = 524288
METHOD_CONFIGS = {
    "gdn_hybrid_swa": (dict(method="gdn_hybrid_swa", layers=24, width=1536, heads=12, mlp_width=6144,
                            sequence_len=4096, backend="fla_chunk64", sliding_window=2048, window_pattern="L",
                            scale="custom"), 524288),
    "kda_hybrid": (dict(method="kda_hybrid", layers=24, width=1536, heads=12, mlp_width=6144, sequence_len=4096,
                        backend="fla_chunk64", window_pattern="L", scale="custom"), 524288),
    # 16 query heads / 1 KV group of dim 128 at width 1536: q 1536 -> 2048, output 2048 -> 1536
    "nsa": (dict(method="nsa", layers=24, width=1536, heads=16, kv_heads=1, attn_head_dim=128, mlp_width=6144,
                 sequence_len=8192, compression_size=32, compression_stride=16, block_size=64, sparse_topk=1024,
                 local_window=512, window_pattern="L", scale="custom"), 524288),
    "moba": (dict(method="moba", layers=24, width=1536, heads=16, kv_heads=1, attn_head_dim=128, mlp_width=6144,
                  sequence_len=8192, block_size=512, sparse_topk=1536, window_pattern="L", scale="custom"), 524288),
    "moe": (dict(method="moe", layers=16, width=2048, heads=16, kv_heads=4, mlp_width=8192, sequence_len=4096,
                 moe_experts=64, moe_topk=8, moe_ffn=1024, moe_shared=1, window_pattern="L", scale="custom"), 1048576),
}
METRIC = "train tokens/sec on 8\u00d7B200 (max over ranks) per method at matched FLOPs/token"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--micro-batch", type=int, default=0, help="rows per micro-batch (default 32 ours / 16 reference)")
    p.add_argument("--comm", choices=("nccl", "p2p"), default="nccl",
                   help="gradient averaging / parameter gather of our arm on N > 1: NCCL collectives (default) "
                        "or the peer-memory kernels (their standalone checks are exact; the training step "
                        "with them is still being validated)")
    p.add_argument("--breakdown", action="store_true",
                   help="also report per-rank CUDA-event phase times (forward+backward, optimizer) of the timed "
                        "updates")
    p.add_argument("--overlap", action="store_true",
                   help="N > 1: start each layer's gradient reductions during the last backward and let the next "
                        "forward wait for each layer's parameter gathers (default: grouped reductions after the "
                        "backward)")
    p.add_argument("--method", default="dense", choices=("dense", *METHOD_CONFIGS),
                   help="benchmark configuration (default: the dense headline configuration)")
    p.add_argument("--layers", type=int, default=MODEL["n_layer"], help=argparse.SUPPRESS)
    p.add_argument("--no-e2e", action="store_true", help=argparse.SUPPRESS)
    return p.parse_args()


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region (local rank 0 only)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled):
        self.proc = None
        self.enabled = enabled

    def __enter__(self):
        if self.enabled:
            try:
                self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                              "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                             text=True)
            except OSError:
                self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self, gpus):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in gpus:
                continue
            rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        seen = set()
        mhz = []
        for r in rows:
            try:
                mhz.append(float(r[1]))
            except ValueError:
                pass
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    seen.add(name)
        try:
            mx = float(rows[0][2])
        except ValueError:
            mx = None
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(seen),
                "samples": len(rows)}


def synthetic_batches(n_micro, rows, T, vocab, seed, device=None, pinned=False):
    import torch
    g = torch.Generator().manual_seed(seed)
    xs, ys = [], []
    for _ in range(n_micro):
        tok = torch.randint(0, vocab, (rows, T + 1), generator=g)
        x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
        if pinned:
            x, y = x.pin_memory(), y.pin_memory()
        if device is not None:
            x, y = x.to(device), y.to(device)
        xs.append(x)
        ys.append(y)
    return xs, ys


def count_own_kernels(step_fn, optimizer=None):
    """Launches of this repository's kernels in one step (torch profiler, outside the timed region).
    The step runs without the data-parallel overlap: no collective is issued from the autograd thread
    while the profiler is active."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    saved = None
    if optimizer is not None and getattr(optimizer, "defer_gathers", False):
        optimizer.flush()
        saved = optimizer.overlap_off()
    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step_fn()
            torch.cuda.synchronize()
    finally:
        if saved is not None:
            optimizer.overlap_restore(saved)
    n = 0
    for ev in prof.events():
        name = ev.name or ""
        if ev.device_type == torch.autograd.DeviceType.CUDA and (name.startswith("void nt::") or "nt::" in name[:40]):
            n += 1
    return n


def timed_steps(step_fn, xs, ys, steps, world, device, flush=None):
    import torch
    import torch.distributed as dist
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize()
    start.record()
    out = None
    for _ in range(steps):
        out = step_fn(xs, ys)
    if flush is not None:
        flush()     # the last update's parameter gathers belong to the timed work
    end.record()
    if world > 1:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end) / steps], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), out


def bench_method(args, rank, world, local, device):
    """One survey benchmark configuration on the generic model path (ours or the reference's)."""
    import torch
    from nexttransformer_b200.runtime.process import shutdown
    raw, global_batch = METHOD_CONFIGS[args.method]
    T = raw["sequence_len"]
    per_rank = global_batch // world
    # rows per micro-batch: activations of 32k tokens per pass (8k for the 64-expert MoE)
    micro = args.micro_batch or max(1, min((8192 if raw["method"] == "moe" else 32768) // T, per_rank // T))
    accum = per_rank // (micro * T)
    try:
        if args.impl == "ours":
            from nexttransformer_b200.models.lm import build_model
            from nexttransformer_b200.optim.groups import protocol_groups
            from nexttransformer_b200.optim.muon_adamw import MuonAdamW
            from nexttransformer_b200.training.engine import Trainer
            from dataclasses import replace
            from nexttransformer_b200.models.config import candidate_config
            config = replace(candidate_config(raw["method"]), **{k: v for k, v in raw.items() if k != "method"})
            model = build_model(config, device, seed=42)
            if raw["method"] in ("nsa", "moba"):
                model.set_sparse_backend("kernel")      # block-sparse sm_100a kernels
            if raw["method"] == "moe" and world > 1:
                from nexttransformer_b200.parallel.expert import enable_expert_parallel
                enable_expert_parallel(model)
            shadows = {p: s for p, s in model.fused_state().casts}
            opt = MuonAdamW(protocol_groups(model), shadows=shadows)
            if world > 1 and args.overlap and model.fused_supported():
                opt.overlap_with(model)
            trainer = Trainer(model, opt, accumulation=accum)
            step_device, step_e2e = trainer.step_device, trainer.step
            flush = trainer.flush
        else:
            from dataclasses import replace
            from nexttransformer.models import build_model as ref_build
            import nexttransformer.models.config as rc
            fields = rc.ModelConfig.__dataclass_fields__
            missing = sorted(k for k in raw if k not in fields and k != "scale")
            if missing:
                raise NotImplementedError(f"the reference's ModelConfig has no {', '.join(missing)} "
                                          f"(this configuration needs them)")
            # the reference admits only formal (d24 shell) and debug scales; debug takes any dimensions
            config = replace(rc.candidate_config(raw["method"]),
                             **{k: v for k, v in raw.items() if k not in ("method", "scale")}, scale="debug")
            model = ref_build(config, device)
            try:
                # the optimizer of the reference's own trainer (train.py): method-auxiliary and
                # non-matrix parameters to AdamW, matrices by shape to Muon
                from nexttransformer.training.optimizer import build_optimizer as ref_optimizer
                from nexttransformer.models.native.config import NativeTrainConfig
                opt = ref_optimizer(model, NativeTrainConfig())
            except ImportError:
                opt = model.setup_optimizer() if hasattr(model, "setup_optimizer") else None
            if opt is None:
                raise RuntimeError("the reference model exposes no optimizer setup")

            def step_device(xs, ys):
                tot = torch.zeros((), device=device)
                for x, y in zip(xs, ys):
                    loss = model(x, y)
                    (loss / accum).backward()
                    tot += loss.detach()
                opt.step()
                model.zero_grad(set_to_none=True)
                return tot / accum

            def step_e2e(xs, ys):
                return float(step_device([x.to(device, non_blocking=True) for x in xs],
                                         [y.to(device, non_blocking=True) for y in ys]))

            def flush():
                pass
        vocab = raw.get("vocab_size", 32768)
        dev_x, dev_y = synthetic_batches(accum, micro, T, vocab, seed=1000 + rank, device=device)
        host_x, host_y = synthetic_batches(accum, micro, T, vocab, seed=2000 + rank, pinned=True)
        for _ in range(args.warmup):
            step_device(dev_x, dev_y)
        flush()
        sampler = ClockSampler(local == 0)
        with sampler:
            ms, loss = timed_steps(step_device, dev_x, dev_y, args.steps, world, device, flush)
        e2e = None
        if not args.no_e2e:
            ms2, _ = timed_steps(step_e2e, host_x, host_y, args.steps, world, device, flush)
            h2d = sum(x.numel() * x.element_size() + y.numel() * y.element_size() for x, y in zip(host_x, host_y))
            e2e = {"value": global_batch / (ms2 / 1000.0), "unit": "tokens/s", "ms_per_step": ms2,
                   "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": 4}
        launches = None
        if args.impl == "ours":
            try:
                launches = count_own_kernels(lambda: (step_device(dev_x, dev_y), flush()), opt) * args.steps
            except Exception:
                launches = None
    except Exception as exc:
        if args.impl != "reference":
            raise
        if rank == 0:
            print(json.dumps({"impl": "reference", "method": args.method,
                              "unavailable": f"{type(exc).__name__}: {exc}"[:300]}), flush=True)
        shutdown()
        return
    value = global_batch / (ms / 1000.0)
    gpus = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", ",".join(str(i) for i in range(world))).split(",")
            if x.strip().isdigit()] or list(range(world))
    clocks = sampler.summary(set(gpus[:world]) if local == 0 else set())
    if rank == 0:
        par = f"dp{world}" + (f"+ep{world}" if raw["method"] == "moe" and world > 1 else "")
        out = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
               "vs_baseline": None, "dtype": "bf16", "data": "synthetic uniform tokens, random-init weights",
               "config": {"model": args.method, "method_config": raw, "global_batch": global_batch, "seq_len": T,
                          "parallelism": par, "micro_batch": micro, "grad_accum": accum,
                          "l2": "working set >> L2 (no flush needed)"},
               "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "loss": float(loss)}
        if args.impl == "reference":
            out["impl"] = "reference"
            out.pop("gpu_launches")
        print(json.dumps(out), flush=True)
    del model
    shutdown()


def main():
    args = parse()
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun for N > 1")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        ref = ROOT / "baseline" / "_ref"
        if not (ref / "nanochat").is_dir():
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
            return
        sys.path.append(str(ref))

    from nexttransformer_b200.runtime.process import initialize, shutdown
    rank, world, device = initialize(seed=42, timeout_s=300)
    if device.type != "cuda":
        raise SystemExit("bench.py needs a CUDA device")
    if args.method != "dense":
        return bench_method(args, rank, world, local, device)
    micro = args.micro_batch or (32 if args.impl == "ours" else 16)
    T = MODEL["sequence_len"]
    per_rank = GLOBAL_BATCH // world
    if per_rank % (micro * T):
        micro = max(1, per_rank // T)
    accum = per_rank // (micro * T)
    cfg = dict(MODEL, n_layer=args.layers)

    if args.impl == "ours":
        from nexttransformer_b200.models.shell import ShellConfig, build_shell
        from nexttransformer_b200.optim.groups import shell_groups
        from nexttransformer_b200.optim.muon_adamw import MuonAdamW
        from nexttransformer_b200.training.engine import Trainer
        model = build_shell(ShellConfig(**cfg), device, seed=42)
        p2p = world > 1 and args.comm == "p2p"
        if p2p:
            from nexttransformer_b200.parallel.symmetric import (PeerReduceScatter, fused_state_with_arena,
                                                                 ownership_segments)
            try:
                st = fused_state_with_arena(model, dist.group.WORLD)
            except Exception as exc:  # symmetric memory unavailable: NCCL collectives instead
                if rank == 0:
                    print(f"peer-memory gradients unavailable ({exc}); using NCCL", file=sys.stderr)
                p2p, args.comm = False, "nccl"
                model._fused = None
        if not p2p:
            st = model.fused_state()
        opt = MuonAdamW(shell_groups(model), shadows={p: s for p, s in st.casts})
        if p2p:
            from nexttransformer_b200.parallel.symmetric import ParamArena, PeerParamGather, param_segments
            segs, covered = ownership_segments(opt, st.arena, world)
            opt.use_peer_reduce_scatter(PeerReduceScatter(st.arena, segs, rank, world), covered)
            if os.environ.get("NT_P2P_GATHER", "0") == "1":
                psegs = param_segments(opt, st.arena, world)
                gather = PeerParamGather(ParamArena(st.arena, psegs, dist.group.WORLD), psegs,
                                         {p: s for p, s in st.casts}, rank, world)
                opt.use_peer_gather(gather, gather.covered)
                if rank == 0:
                    print(f"peer-memory step: reduce-scatter pad {int(opt.p2p.pads[rank]):#x}, gather pad "
                          f"{int(gather.pads[rank]):#x}, {len(segs)} segments, {opt.p2p.blocks} / {gather.blocks} "
                          f"blocks", file=sys.stderr)
        overlap = world > 1 and args.overlap
        if overlap:
            opt.overlap_with(model)
        trainer = Trainer(model, opt, accumulation=accum)

        def step_device(xs, ys):
            return trainer.step_device(xs, ys)

        def step_e2e(xs, ys):
            return trainer.step(xs, ys)
        flush = trainer.flush
        flops_per_token = model.estimate_flops()
    else:
        from nexttransformer.models.backbone import GPT, GPTConfig
        with torch.device("meta"):
            model = GPT(GPTConfig(**cfg))
        model.to_empty(device=device)
        model.init_weights()
        opt = model.setup_optimizer()

        def step_device(xs, ys):
            tot = torch.zeros((), device=device)
            for x, y in zip(xs, ys):
                loss = model(x, y)
                (loss / accum).backward()
                tot += loss.detach()
            opt.step()
            model.zero_grad(set_to_none=True)
            return tot / accum

        def step_e2e(xs, ys):
            return float(step_device([x.to(device, non_blocking=True) for x in xs],
                                     [y.to(device, non_blocking=True) for y in ys]))

        def flush():
            pass
        overlap = False
        flops_per_token = model.estimate_flops()

    vocab = MODEL["vocab_size"]
    dev_x, dev_y = synthetic_batches(accum, micro, T, vocab, seed=1000 + rank, device=device)
    host_x, host_y = synthetic_batches(accum, micro, T, vocab, seed=2000 + rank, pinned=True)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[device.index])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step_device(dev_x, dev_y)
    flush()
    barrier()

    # ---- device-timed region
    if args.breakdown and args.impl == "ours":
        trainer.timing = True
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local == 0)
    with sampler:
        barrier()
        start.record()
        for _ in range(args.steps):
            loss = step_device(dev_x, dev_y)
        flush()     # the last update's parameter gathers belong to the timed work
        end.record()
        barrier()
    ms = start.elapsed_time(end) / args.steps
    breakdown = None
    if args.breakdown and args.impl == "ours":
        trainer.timing = False
        phases = trainer.phase_times()
        mine = torch.tensor([statistics.median(p[0] for p in phases), statistics.median(p[1] for p in phases), ms],
                            device=device, dtype=torch.float64)
        every = [torch.empty_like(mine) for _ in range(world)] if world > 1 else [mine]
        if world > 1:
            dist.all_gather(every, mine)
        breakdown = [{"rank": r, "forward_backward_ms": float(t[0]), "optimizer_ms": float(t[1]),
                      "step_ms": float(t[2])} for r, t in enumerate(every)]
    if rank == 0:
        print(f"timed region done: {ms:.1f} ms per step", file=sys.stderr, flush=True)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    final_loss = float(loss)

    # ---- end-to-end through the public step call (H2D of inputs, D2H of the loss)
    e2e = None
    if not args.no_e2e:
        for _ in range(1):
            step_e2e(host_x, host_y)
        flush()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            step_e2e(host_x, host_y)
        flush()
        e2.record()
        barrier()
        ms2 = s2.elapsed_time(e2) / args.steps
        t2 = torch.tensor([ms2], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        ms2 = float(t2.item())
        h2d = sum(x.numel() * x.element_size() + y.numel() * y.element_size() for x, y in zip(host_x, host_y))
        e2e = {"value": GLOBAL_BATCH / (ms2 / 1000.0), "unit": "tokens/s", "ms_per_step": ms2,
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": 4}

    if rank == 0:
        print("end-to-end region done", file=sys.stderr, flush=True)
    # every rank must hold the same parameters after the updates (checks the parameter all-gather)
    params_agree = None
    flush()
    if world > 1:
        digest = torch.stack([sum(p.detach().double().sum() for p in model.parameters()),
                              sum(p.detach().double().abs().sum() for p in model.parameters())])
        all_d = [torch.empty_like(digest) for _ in range(world)]
        dist.all_gather(all_d, digest)
        params_agree = all(bool(torch.equal(d, all_d[0])) for d in all_d)

    launches = None
    if args.impl == "ours":
        barrier()       # every rank enters the profiled step together (its peer-memory kernels wait on peers)
        try:
            launches = count_own_kernels(lambda: (step_device(dev_x, dev_y), flush()), opt) * args.steps
        except Exception as exc:  # profiler unavailable: report as unknown
            launches = None
            if rank == 0:
                print(f"launch count unavailable: {exc}", file=sys.stderr)

    value = GLOBAL_BATCH / (ms_max / 1000.0)
    gpus = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", ",".join(str(i) for i in range(world))).split(",")
            if x.strip().isdigit()] or list(range(world))
    clocks = sampler.summary(set(gpus[:world]) if local == 0 else set())
    if rank == 0:
        out = {"metric": METRIC,
               "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
               "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None, "dtype": "bf16",
               "data": "synthetic uniform tokens, random-init weights",
               "config": {"model": "dense GQA d20 w1280 h10/kv5 hd128 vocab65536 (shell: VE, smear, backout, softcap)",
                          "global_batch": GLOBAL_BATCH, "seq_len": T, "parallelism": f"dp{world}",
                          "micro_batch": micro, "grad_accum": accum, "l2": "working set >> L2 (no flush needed)",
                          "grad_comm": (args.comm if world > 1 else "none") if args.impl == "ours" else "nccl",
                          "overlap": overlap,
                          "param_gather": ("p2p" if args.comm == "p2p" and os.environ.get("NT_P2P_GATHER", "0") == "1"
                                           else "nccl") if world > 1 and args.impl == "ours"
                          else ("none" if world == 1 else "nccl"),
                          "flops_per_token": flops_per_token, "params_equal_across_ranks": params_agree},
               "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "loss": final_loss}
        if breakdown is not None:
            out["phase_breakdown"] = breakdown
        if args.impl == "reference":
            out["impl"] = "reference"
            out.pop("gpu_launches")
        print(json.dumps(out), flush=True)
    # symmetric-memory buffers (the peer path) are released after the process group, never while a
    # peer may still be tearing down its mappings
    barrier()
    shutdown()
    del opt, model


if __name__ == "__main__":
    main()
