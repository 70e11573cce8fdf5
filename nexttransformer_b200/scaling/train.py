"""Dense scaling-stage pretraining on nodes that share no filesystem:
``python -m nexttransformer_b200.scaling.train --config configs/scaling/<name>.json``.

``--dry-run`` prints the plan, ``--benchmark STEPS`` times updates, ``--smoke-steps`` runs a bounded
test that is never a completed pretraining run.  Before training every rank compares its source
files, configuration, data identity and software versions with every other rank; each node writes
its own checkpoints and status file, rank zero the event history.  Gradients go to their owners
through the Muon/AdamW optimizer's reduce-scatter (no DDP wrapper, no full gradient all-reduce).
A first SIGTERM / SIGINT or an ``output/STOP`` file stops every rank after the current update with
a checkpoint; a non-finite loss or gradient exits with code 3 (restarting would replay it).
Behaviour: ``nexttransformer/scaling/train.py:103-373`` of the reference.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
from dataclasses import asdict, replace
from functools import partial
import hashlib
import json
import os
from pathlib import Path
import signal
import socket
import statistics
import sys
import time

import torch
import torch.distributed as dist
from torch.utils.checkpoint import checkpoint

NONFINITE_EXIT = 3
# Dense bf16 tensor-core peaks for the reported MFU; a name is matched before its substrings.
PEAK_FLOPS = (("B200", 2250e12), ("H200", 989e12), ("H100", 989e12), ("H800", 989e12), ("H20", 148e12),
              ("A100", 312e12), ("A800", 312e12), ("L40S", 362e12))
_stop_signal = []


def peak_flops(device):
    if device.type != "cuda":
        return None
    name = torch.cuda.get_device_name(device)
    return next((peak for key, peak in PEAK_FLOPS if key in name), None)


def source_manifest():
    """sha256 over every source file of the package (Python, CUDA, C++), by relative path."""
    root = Path(__file__).resolve().parents[1]
    files = {}
    for path in sorted(root.rglob("*")):
        if path.is_file() and path.suffix in (".py", ".cu", ".cuh", ".h", ".cpp") and "__pycache__" not in path.parts:
            files[str(path.relative_to(root))] = hashlib.sha256(path.read_bytes()).hexdigest()
    blob = json.dumps(files, sort_keys=True).encode()
    return {"sha256": hashlib.sha256(blob).hexdigest(), "files": len(files)}


def check_nodes(identity):
    """Every rank runs the same sources, software, configuration and data; returns {node: host}."""
    from nexttransformer_b200.scaling.checkpoint import gather, topology
    node, _, _ = topology()
    entries = gather({"node": node, "host": socket.gethostname(), **identity})
    for key in identity:
        seen = {}
        for e in entries:
            seen.setdefault(json.dumps(e[key], sort_keys=True), set()).add(e["host"])
        if len(seen) > 1:
            raise ValueError(f"nodes disagree on {key}: " + "; ".join(f"{sorted(h)} {v}" for v, h in seen.items()))
    return {f"{e['node']:03d}": e["host"] for e in entries}


def _request_stop(number, frame):
    # The first signal stops after the current update with a checkpoint; a second one ends at once.
    _stop_signal.append(number)
    signal.signal(number, signal.SIG_DFL)


def archive_records(output):
    """Move the records of a run that never reached a checkpoint aside before it restarts at step 0."""
    archive = Path(output) / "restarts" / str(time.time_ns())
    for path in Path(output).iterdir():
        if path.is_file() and path.suffix in (".json", ".jsonl") and not path.name.startswith("status.node"):
            archive.mkdir(parents=True, exist_ok=True)
            try:
                path.rename(archive / path.name)
            except FileNotFoundError:
                pass


def rewind_events(output, step):
    """Keep the event history up to `step`; later events move to metrics.after_<step>.jsonl."""
    path = Path(output) / "metrics.jsonl"
    if not path.exists():
        return
    keep, later = [], []
    for line in path.read_text().splitlines():
        (keep if json.loads(line).get("step", 0) <= step else later).append(line)
    if later:
        (Path(output) / f"metrics.after_{step:08d}.jsonl").write_text("\n".join(later) + "\n")
    path.write_text("".join(line + "\n" for line in keep))


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    p.add_argument("--config", required=True, type=Path)
    p.add_argument("--output", type=Path)
    p.add_argument("--world-size", type=int, default=32, help="dry-run planning only; runtime uses WORLD_SIZE")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--resume", default="never", help="never | auto | <step>")
    p.add_argument("--allow-source-change", action="store_true", help="resume with changed source files (recorded)")
    p.add_argument("--data", choices=("bestfit", "synthetic"), default="synthetic")
    p.add_argument("--prefetch", type=int, default=2,
                   help="micro-batches packed ahead on a background thread (real data; 0: pack inline)")
    p.add_argument("--smoke-steps", type=int, default=0, help="short test, never a completed pretraining run")
    p.add_argument("--smoke-val-tokens", type=int, default=0, help="0: one distributed evaluation batch")
    p.add_argument("--stop-after", type=int, default=0, help="checkpoint and stop after this many updates")
    p.add_argument("--benchmark", type=int, default=0, metavar="STEPS", help="time STEPS updates, write nothing")
    p.add_argument("--benchmark-batch-tokens", type=int, default=0, help="benchmark-only global batch")
    p.add_argument("--log-every", type=int, default=10)
    p.add_argument("--recompute-layers", type=int, default=0,
                   help="recompute the first N blocks in the backward (-1: every block)")
    p.add_argument("--bf16-grad-reduce", action="store_true", help="reduce gradients in bf16")
    p.add_argument("--keep-local", type=int, default=3, help="rolling checkpoints kept per node besides milestones")
    p.add_argument("--core", type=Path, help="CORE bundle (tasks.json + <label>.jsonl): evaluated at the core steps")
    p.add_argument("--tokenizer", type=Path, help="tokenizer directory for CORE (default: RESOURCES/tokenizer)")
    from nexttransformer_b200.evaluation.context import add_core_max_tokens
    add_core_max_tokens(p)
    a = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(a)
    a.micro_batch = int(a.micro_batch or 2)
    if a.log_every < 1:
        p.error("--log-every must be positive")
    if a.resume not in ("never", "auto") and not a.resume.isdigit():
        p.error("--resume takes never, auto or a step")
    if a.benchmark and (a.smoke_steps or a.stop_after or a.resume != "never"):
        p.error("--benchmark cannot be combined with smoke, stop or resume options")
    if a.benchmark_batch_tokens and not a.benchmark:
        p.error("--benchmark-batch-tokens needs --benchmark")
    if a.keep_local < 2:
        p.error("--keep-local must keep at least two checkpoints")
    return a


def plan(mc, tc, world, micro):
    from nexttransformer_b200.models.native.model import NativeExperiment, theoretical_training_flops
    from nexttransformer_b200.scaling.config import config_hash
    from nexttransformer_b200.scaling.optimizer import muon_weight_decay, scaling_params
    with torch.device("meta"):
        model = NativeExperiment(mc)
    flops = theoretical_training_flops(mc)
    return {"model": asdict(mc), "train": asdict(tc), "config_sha256": config_hash(mc, tc),
            "parameters": sum(p.numel() for p in model.parameters()), "scaling_parameters": scaling_params(model),
            "muon_lr": tc.muon_lr * tc.batch_scale, "muon_weight_decay": muon_weight_decay(model, tc),
            "steps": tc.steps, "accumulation": tc.accumulation(mc, world, micro),
            "validation_events": len(tc.validation_steps()), "core_steps": tc.core_steps(),
            "train_GFLOPs_per_input_token": flops / 1e9, "total_training_flops": flops * tc.total_tokens}


def main(argv=None):
    args = parse(argv)
    from nexttransformer_b200.scaling.config import config_hash, load_config
    mc, tc = load_config(args.config)
    if args.benchmark_batch_tokens:
        tc = replace(tc, global_batch_tokens=args.benchmark_batch_tokens,
                     total_tokens=args.benchmark_batch_tokens * tc.steps)
    if args.dry_run:
        print(json.dumps(plan(mc, tc, args.world_size, args.micro_batch), indent=2))
        return None

    from nexttransformer_b200.evaluation.bpb import evaluate_stream_loss
    from nexttransformer_b200.models.native.model import build_model
    from nexttransformer_b200.native.optimizer import clip_halter_gradients, set_schedule
    from nexttransformer_b200.native.train import _LossView, make_stream
    from nexttransformer_b200.optim.muon_adamw import grad_of
    from nexttransformer_b200.runtime.files import atomic_json
    from nexttransformer_b200.runtime.process import append_event, initialize, reduce_max, reduce_sum, synchronize
    from nexttransformer_b200.runtime.statistics import accumulate_stats, training_stats
    from nexttransformer_b200.scaling import checkpoint as ck
    from nexttransformer_b200.scaling.optimizer import build_optimizer, muon_weight_decay, scaling_params

    benchmark = bool(args.benchmark)
    smoke = benchmark or bool(args.smoke_steps)
    output = args.output or Path(args.runtime_dir) / "runs" / (args.run_name or "scaling_" + args.config.stem)
    for number in (signal.SIGTERM, signal.SIGINT):
        signal.signal(number, _request_stop)
    if int(os.environ.get("RANK", "0")) == 0 and not benchmark:
        from nexttransformer_b200.runtime.tracking_auth import preflight
        preflight(args.wandb_mode)
    rank, world, device = initialize(tc.seed)
    node, local_rank, _ = ck.topology()
    accumulation = tc.accumulation(mc, world, args.micro_batch)
    lock = None
    if not benchmark and local_rank == 0:
        import fcntl
        output.mkdir(parents=True, exist_ok=True)
        lock = (output / f"run.node{node:03d}.lock").open("a")
        fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
    if world > 1:
        dist.barrier()
    stream = make_stream(args, mc, rank, world, tc.seed)
    if args.data == "bestfit" and args.prefetch > 0:
        from nexttransformer_b200.runtime.prefetch import PrefetchStream
        stream = PrefetchStream(stream, args.prefetch)
    described = {"kind": args.data, "vocab": mc.vocab_size, "seq": mc.sequence_len, "seed": tc.seed, "world": world}
    if args.data == "bestfit":
        # every node must hold the same shards and the same tokenizer
        from nexttransformer_b200.runtime.resources import data_inventory, inventory_fingerprint, tokenizer_fingerprint
        described.update(inventory=inventory_fingerprint(data_inventory(args.data_dir or Path(args.resources)
                                                                        / "base_data_climbmix")),
                         tokenizer=tokenizer_fingerprint(args.resources))
    data_identity = hashlib.sha256(json.dumps(described, sort_keys=True).encode()).hexdigest()
    source = source_manifest()
    identity = dict(source_sha256=source["sha256"], data=data_identity, config_sha256=config_hash(mc, tc),
                    torch=torch.__version__, cuda=torch.version.cuda)
    hosts = check_nodes(identity)

    resumed = None
    if not benchmark:
        if args.resume == "never":
            if not ck.agree(not (output / "provenance.json").exists(), device):
                raise ValueError("output already contains a run; use --resume auto or a new --output directory")
        else:
            resumed = ck.common_step(output) if args.resume == "auto" else int(args.resume)
            if resumed is not None and not ck.agree(resumed in ck.complete_steps(output, node), device):
                raise ValueError(f"checkpoint {resumed} is not complete on every node")
            if local_rank == 0:
                ck.set_aside_after(output, resumed, node)
                if resumed is None:
                    archive_records(output)
        if world > 1:
            dist.barrier()

    stop_step = min(tc.steps, args.benchmark or args.smoke_steps) if smoke else tc.steps
    batch_tokens = args.micro_batch * world * mc.sequence_len
    val_tokens = (args.smoke_val_tokens or batch_tokens) if smoke else tc.val_tokens
    if val_tokens % batch_tokens:
        raise ValueError("validation tokens must divide the distributed evaluation batch")
    model = build_model(mc, device, seed=tc.seed)
    recompute = len(model.transformer.h) if args.recompute_layers < 0 else min(args.recompute_layers,
                                                                                 len(model.transformer.h))
    for block in model.transformer.h[:recompute]:
        block.forward = partial(checkpoint, block.forward, use_reentrant=False)
    # On CUDA the dense model trains through the fused sm_100a path (it keeps every activation, so
    # not with recompute): the optimizer writes the bf16 shadows the fused forward reads.
    fused = device.type == "cuda" and not recompute and mc.architecture == "dense" and model.fused_supported()
    shadows = None
    if fused:
        shadows = {p: s for p, s in model.fused_state().casts}
        model.use_fused = True
    optimizer = build_optimizer(model, tc, shadows=shadows, bf16_reduce=args.bf16_grad_reduce)
    state = dict(step=0, input_tokens=0, next_global_sequence=0, training_flops_estimate=0.,
                 training_seconds=0., validation_seconds=0., completed_val_steps=[], data=identity["data"])
    if resumed is not None:
        saved = ck.load_checkpoint(output, resumed, model, optimizer, stream, device)
        if fused:
            model.refresh_shadows()
        if not mc.matches(saved["model_config"]) or saved["train_config"] != asdict(tc):
            raise ValueError("resume configuration differs from checkpoint")
        state = saved["state"]
        if state["data"] != identity["data"]:
            raise ValueError("resume data differs from checkpoint")
        if state["input_tokens"] != state["step"] * tc.global_batch_tokens or \
                state["next_global_sequence"] != state["input_tokens"] // mc.sequence_len:
            raise ValueError("checkpoint token cursor is inconsistent")
        if stream.rows * world * mc.sequence_len != state["input_tokens"]:
            raise ValueError("rank-local data cursor differs from checkpoint token count")
        if state.get("smoke", False) != smoke:
            raise ValueError("smoke checkpoints cannot be promoted to pretraining runs")
        if state["source_sha256"] != source["sha256"] and not args.allow_source_change:
            raise ValueError("resume source files differ from checkpoint; pass --allow-source-change")
        del saved
        from nexttransformer_b200.evaluation.context import resume_core_limit
        args.core_max_tokens = resume_core_limit(state, args.core_max_tokens, mc.sequence_len)
    state["core_max_tokens"] = args.core_max_tokens
    tasks, tokenizer = None, None
    if args.core and not benchmark:
        from nexttransformer_b200.evaluation.context import check_full_context
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tasks = json.loads((args.core / "tasks.json").read_text())
        for t in tasks:
            t["data"] = [json.loads(l) for l in (args.core / f"{t['label']}.jsonl").read_text().splitlines() if l]
        tokenizer = BPETokenizer.from_directory(args.tokenizer or Path(args.resources) / "tokenizer")
        if tokenizer.get_vocab_size() > mc.vocab_size:
            raise ValueError("the tokenizer's vocabulary does not fit the model")
        if not smoke:
            check_full_context(mc, args.core_max_tokens)
    previous_source = state.get("source_sha256")
    state["source_sha256"], state["smoke"] = source["sha256"], smoke
    if not benchmark and rank == 0:
        if resumed is not None:
            rewind_events(output, state["step"])
        atomic_json(output / ("provenance.json" if resumed is None else f"resume_{state['step']:08d}.json"), {
            "model": asdict(mc), "train": asdict(tc), **identity, "source": source,
            "previous_source_sha256": previous_source, "command": sys.argv, "world_size": world, "nodes": hosts,
            "device": torch.cuda.get_device_name(device) if device.type == "cuda" else str(device),
            "micro_batch": args.micro_batch, "gradient_accumulation": accumulation, "recompute_layers": recompute,
            "fused_path": fused,
            "bf16_grad_reduce": args.bf16_grad_reduce, "smoke": smoke,
            "parameters": sum(p.numel() for p in model.parameters()), "scaling_parameters": scaling_params(model),
            "muon_weight_decay": muon_weight_decay(model, tc)})
    peak = peak_flops(device)

    def record(event):
        if rank == 0 and not benchmark:
            append_event(output, event)
            print(json.dumps(event), flush=True)

    def core(step, final=False):
        from nexttransformer_b200.evaluation.context import LengthProbe, core_context, inference_view
        from nexttransformer_b200.evaluation.core import evaluate_core
        model.eval()          # before the view is taken: the shallow copy keeps the mode it was made in
        probe = LengthProbe(inference_view(model, args.core_max_tokens))
        with torch.no_grad():
            result = evaluate_core(probe, tokenizer, tasks, device, rank, world,
                                   -1 if final else tc.core_max_per_task, args.core_max_tokens)
        model.train()
        longest = torch.tensor(probe.longest, device=device)
        if world > 1:
            dist.all_reduce(longest, op=dist.ReduceOp.MAX)
        result["coreContext"] = core_context(mc.sequence_len, args.core_max_tokens, int(longest.item()))
        record({"event": "core", "step": step, **result})
        if rank == 0:
            atomic_json(output / ("core_final.json" if final else f"core_{step:08d}.json"),
                        {"event": "core", "step": step, **result})

    def evaluate(tokens, seed_offset=0):
        """Bits per byte on the validation split with real data; the held-out synthetic stream's loss
        otherwise."""
        if args.data == "synthetic":
            return evaluate_stream_loss(_LossView(model), mc, tokens, args.micro_batch, rank, world, device,
                                        tc.seed + seed_offset)
        from nexttransformer_b200.evaluation.bpb import evaluate_bpb
        from nexttransformer_b200.runtime.data import BestFitStream
        t0 = time.time()
        val = BestFitStream(args.data_dir or Path(args.resources) / "base_data_climbmix", stream.tokenizer, "val",
                            rank, world, mc.sequence_len)
        steps = max(1, tokens // (world * args.micro_batch * mc.sequence_len))
        bpb = evaluate_bpb(_LossView(model), val.batches(args.micro_batch, device), steps,
                           stream.tokenizer.token_bytes().to(device))
        return {"val_bpb": bpb, "val_tokens": steps * world * args.micro_batch * mc.sequence_len,
                "seconds": time.time() - t0}

    def validation(step):
        if benchmark or step in state["completed_val_steps"]:
            return
        result = evaluate(val_tokens)
        state["completed_val_steps"].append(step)
        state["validation_seconds"] += result["seconds"]
        record({"event": "validation", "step": step, **result})
        if rank == 0:
            atomic_json(output / f"val_{step:08d}.json", {"event": "validation", "step": step, **result})

    model.train()
    if state["step"] == 0:
        validation(0)
    phase, launched, timings, last_checkpoint = None, state["step"], [], None
    for step in range(state["step"], stop_step):
        synchronize(device)
        start, data_seconds = time.perf_counter(), 0.
        if device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(device)
        optimizer.zero_grad(set_to_none=True)
        if fused:
            model.zero_main_grads()
        scale = set_schedule(optimizer, step, tc)
        stats = training_stats(mc, device)
        for _ in range(accumulation):
            t = time.perf_counter()
            x, y = stream.batch(args.micro_batch, device)
            data_seconds += time.perf_counter() - t
            out = model(x, y)
            (out["loss"] / accumulation).backward()
            accumulate_stats(stats, out, model.last_stats, accumulation, world, mc)
        # every rank sees the same verdict, so all ranks stop together
        gsq = torch.zeros((), device=device, dtype=torch.float64)
        for p in model.parameters():
            g = grad_of(p)
            if g is not None:
                gsq += g.double().square().sum()
        bad = torch.tensor([0. if torch.isfinite(gsq) and torch.isfinite(stats).all() else 1.], device=device)
        reduce_max(bad)
        if bad.item():
            values = reduce_sum(stats).tolist()
            record({"event": "nonfinite", "step": step + 1, "lm_loss": values[0]})
            phase = "nonfinite"
            break
        grad_norm = float(gsq.sqrt())
        if tc.grad_clip:
            torch.nn.utils.clip_grad_norm_(model.parameters(), tc.grad_clip)
        clip_halter_gradients(model)
        synchronize(device)
        optimizer_start = time.perf_counter()
        optimizer.step()
        synchronize(device)
        optimizer_seconds = time.perf_counter() - optimizer_start
        values = reduce_sum(stats).tolist()
        if int(values[4]) != tc.global_batch_tokens:
            raise RuntimeError("training input-token budget drift")
        duration = time.perf_counter() - start
        state["step"] = step + 1
        state["input_tokens"] += tc.global_batch_tokens
        state["next_global_sequence"] = state["input_tokens"] // mc.sequence_len
        state["training_flops_estimate"] += values[2]
        state["training_seconds"] += duration
        memory = torch.cuda.max_memory_allocated(device) if device.type == "cuda" else 0
        timings.append((duration, data_seconds, optimizer_seconds, memory, values[2]))
        if (step + 1) % args.log_every == 0 or step == launched or step + 1 == stop_step:
            record({"event": "train", "step": step + 1, "input_tokens": state["input_tokens"], "lm_loss": values[0],
                    "loss": values[6 + mc.routing_steps], "grad_norm_local": grad_norm, "lr_multiplier": scale,
                    "step_flops_estimate": values[2], "tokens_per_second": tc.global_batch_tokens / duration,
                    "mfu": values[2] / (duration * world * peak) if peak else None, "step_seconds": duration,
                    "data_seconds": data_seconds, "optimizer_seconds": optimizer_seconds,
                    "gpu_hours": world * state["training_seconds"] / 3600, "peak_memory_bytes": memory})
        if state["step"] % tc.val_every == 0 or state["step"] == stop_step:
            validation(state["step"])
        if tasks is not None and not smoke and state["step"] < tc.steps and state["step"] in tc.core_steps():
            core(state["step"])
        requested = bool(_stop_signal) or (rank == 0 and not benchmark and (output / "STOP").exists())
        stop = not ck.agree(not requested, device) or bool(args.stop_after and state["step"] - launched >= args.stop_after)
        if not benchmark and (state["step"] % tc.checkpoint_every == 0 or state["step"] == stop_step or stop):
            last_checkpoint = ck.save_checkpoint(output, model, optimizer, stream, mc, tc, state,
                                                 milestone=not smoke and tc.is_milestone(state["step"]))
            if local_rank == 0:
                ck.prune(output, node, args.keep_local)
        if stop and state["step"] < stop_step:
            if rank == 0 and (output / "STOP").exists():
                (output / "STOP").rename(output / f"STOP.consumed-{state['step']:08d}")
            phase = "stopped"
            break
    complete = phase is None and not smoke and state["step"] == tc.steps
    if complete:
        # the final checkpoint precedes this evaluation; a restart repeats only the evaluation
        final = evaluate(tc.final_bpb_tokens, 1)
        if rank == 0:
            atomic_json(output / "bpb_final.json", {"step": state["step"], "val": final})
        record({"event": "final_bpb", "step": state["step"], **{"final_" + k: v for k, v in final.items()}})
        if tasks is not None:
            core(state["step"], final=True)
    phase = phase or ("smoke_complete" if smoke else "training_complete" if complete else "stopped")
    if benchmark and timings:
        measured = timings[min(3, len(timings) - 1):]
        memory = torch.tensor(float(max(t[3] for t in measured)), device=device)
        if world > 1:
            dist.all_reduce(memory, op=dist.ReduceOp.MAX)
        seconds = statistics.median(t[0] for t in measured)
        summary = {"event": "benchmark", "world_size": world, "micro_batch": args.micro_batch,
                   "gradient_accumulation": accumulation, "global_batch_tokens": tc.global_batch_tokens,
                   "recompute_layers": recompute, "bf16_grad_reduce": args.bf16_grad_reduce, "fused_path": fused,
                   "measured_steps": len(measured), "step_seconds": seconds,
                   "data_seconds": statistics.median(t[1] for t in measured),
                   "optimizer_seconds": statistics.median(t[2] for t in measured),
                   "tokens_per_second_per_gpu": tc.global_batch_tokens / seconds / world,
                   "mfu": statistics.median(t[4] for t in measured) / (seconds * world * peak) if peak else None,
                   "peak_memory_gib": memory.item() / 2 ** 30}
        if rank == 0:
            print(json.dumps(summary), flush=True)
            if args.output:
                atomic_json(args.output / "benchmark.json", summary)
    elif not benchmark and rank == 0:
        atomic_json(output / "run_status.json", {"phase": phase, **state,
                                                 "checkpoint": str(last_checkpoint) if last_checkpoint else None})
    if not benchmark and local_rank == 0:
        atomic_json(output / f"status.node{node:03d}.json", {"phase": phase, "step": state["step"], "time": time.time()})
    if world > 1:
        dist.destroy_process_group()
    if lock is not None:
        lock.close()
    if phase == "nonfinite":
        sys.exit(NONFINITE_EXIT)
    return state


if __name__ == "__main__":
    main()
