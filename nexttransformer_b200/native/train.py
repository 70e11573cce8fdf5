"""Native d24 comparison trainer: ``python -m nexttransformer_b200.native.train --config configs/native/<arch>.json``.

One process per GPU (torchrun); gradients are reduced to their owners by the Muon/AdamW optimizer.
Per update: curriculum step (Circle) -> schedule -> micro-batches (loss dict: lm + router/budget
penalty) -> accounting vector -> non-finite check -> halter / conditioner clips -> update -> one
all-reduce of the accounting -> route-budget update from the global survival counts -> events,
validation and checkpoints.  ``--dry-run`` prints the plan (parameters, accumulation, FLOPs per
token) without a GPU.  ``--smoke-steps`` runs a short test that is never a completed pretraining run.
Behaviour: ``nexttransformer/native/train.py:35-249``.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
from dataclasses import asdict
import json
from pathlib import Path
import sys
import time

import torch

NONFINITE_EXIT = 3


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    p.add_argument("--config", required=True, type=Path)
    p.add_argument("--output", type=Path)
    p.add_argument("--world-size", type=int, default=8, help="dry-run planning only; runtime uses WORLD_SIZE")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--resume", default="never", help="never | auto")
    p.add_argument("--data", choices=("bestfit", "synthetic"), default="synthetic")
    p.add_argument("--prefetch", type=int, default=2,
                   help="micro-batches packed ahead on a background thread (real data; 0: pack inline)")
    p.add_argument("--smoke-steps", type=int, default=0)
    p.add_argument("--smoke-val-tokens", type=int, default=0)
    p.add_argument("--log-every", type=int, default=10)
    p.add_argument("--checkpoint-every", type=int, default=0, help="0: the configuration's cadence")
    p.add_argument("--circle-stage-step", type=int, default=0, help="smoke-only curriculum offset")
    p.add_argument("--global-batch", type=int, default=0, help="smoke-only override of tokens per update")
    p.add_argument("--seed", type=int, default=None)
    p.add_argument("--core", type=Path, default=None,
                   help="CORE bundle directory (tasks.json + <label>.jsonl) scored at the configuration's CORE steps")
    a = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(a)
    if a.circle_stage_step and not a.smoke_steps:
        p.error("curriculum offset is smoke-only")
    if a.global_batch and not a.smoke_steps:
        p.error("--global-batch is smoke-only")
    if a.log_every < 1:
        p.error("--log-every must be positive")
    return a


def plan(mc, tc, world, micro):
    from nexttransformer_b200.models.native.halter import feature_forward_ops
    from nexttransformer_b200.models.native.model import NativeExperiment, theoretical_training_flops
    with torch.device("meta"):
        m = NativeExperiment(mc)
    return {"model": asdict(mc), "train": asdict(tc), "parameters": sum(p.numel() for p in m.parameters()),
            "accumulation": tc.accumulation(mc, world, micro), "steps": tc.steps,
            "halter_extra_forward_ops_per_input_token": feature_forward_ops(mc),
            "validation_events": len(tc.validation_steps()), "core_steps": tc.core_steps(),
            "train_GFLOPs_per_input_token": theoretical_training_flops(mc) / 1e9}


def data_dir(args):
    return args.data_dir or Path(args.resources) / "base_data_climbmix"


def load_tokenizer(args):
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    return BPETokenizer.from_directory(Path(args.resources) / "tokenizer")


def make_stream(args, mc, rank, world, seed, tok=None):
    from nexttransformer_b200.runtime.data import BestFitStream, SyntheticStream
    if args.data == "synthetic":
        return SyntheticStream(mc.vocab_size, mc.sequence_len, rank, world, seed=seed)
    return BestFitStream(data_dir(args), tok or load_tokenizer(args), "train", rank, world, mc.sequence_len)


def scheduled_evaluations(args, model, tc, tok, tasks, step, final, micro, rank, world, device):
    """Counted BPB at the validation steps and CORE at the CORE steps (real data only), and at the
    end the final train / validation BPB; returns the metric events to log."""
    from nexttransformer_b200.evaluation.native import evaluate_native_bpb, evaluate_native_core
    events = []
    if tok is None:
        return events
    if step in tc.validation_steps():
        res = evaluate_native_bpb(model, tok, data_dir(args), tc.val_tokens, micro, rank, world, device)
        events.append({"event": "validation", "step": step, **res})
    if tasks is not None and step in tc.core_steps():
        res = evaluate_native_core(model, tok, tasks, device, rank, world, tc.core_max_per_task,
                                   model.config.sequence_len)
        events.append({"event": "core", "step": step, **res})
    if final:
        both = {split: evaluate_native_bpb(model, tok, data_dir(args), tc.final_bpb_tokens, micro, rank, world,
                                           device, split) for split in ("train", "val")}
        events.append({"event": "final_bpb", "step": step, "train_bpb": both["train"]["train_bpb"],
                       "val_bpb": both["val"]["val_bpb"], "train": both["train"], "val": both["val"]})
    return events


def update(model, optimizer, stream, mc, tc, accum, micro, world, device, step):
    """One optimizer update; returns the globally reduced accounting vector (None if non-finite)."""
    from nexttransformer_b200.native.optimizer import clip_condition_gradients, clip_halter_gradients
    from nexttransformer_b200.runtime.process import reduce_max, reduce_sum
    from nexttransformer_b200.runtime.statistics import accumulate_stats, training_stats
    from nexttransformer_b200.optim.muon_adamw import grad_of
    optimizer.zero_grad(set_to_none=True)
    if getattr(model, "use_fused", False):
        model.zero_main_grads()
    stats = training_stats(mc, device)
    for _ in range(accum):
        x, y = stream.batch(micro, device)
        out = model(x, y)
        (out["loss"] / accum).backward()
        accumulate_stats(stats, out, model.last_stats, accum, world, mc)
    gsq = torch.zeros((), device=device, dtype=torch.float64)
    for p in model.parameters():
        g = grad_of(p)
        if g is not None:
            gsq += g.double().square().sum()
    bad = torch.tensor([0. if torch.isfinite(gsq) and torch.isfinite(stats).all() else 1.], device=device)
    reduce_max(bad)
    if bad.item():
        return None
    if tc.grad_clip:
        torch.nn.utils.clip_grad_norm_(model.parameters(), tc.grad_clip, error_if_nonfinite=True)
    clip_halter_gradients(model)
    clip_condition_gradients(model)
    optimizer.step()
    reduce_sum(stats)
    values = stats.tolist()
    if int(values[4]) != tc.global_batch_tokens:
        raise RuntimeError("training input-token budget drift")
    model.update_route_budget(values[6:6 + mc.routing_steps], values[4], step)
    return values


def main(argv=None):
    args = parse(argv)
    from dataclasses import replace
    from nexttransformer_b200.models.native.config import load_config
    mc, tc = load_config(args.config)
    if args.global_batch:
        tc = replace(tc, global_batch_tokens=args.global_batch,
                     total_tokens=args.global_batch * max(args.smoke_steps, 1))
    micro = args.micro_batch or 4
    if args.dry_run:
        print(json.dumps(plan(mc, tc, args.world_size, micro), indent=2))
        return None
    from nexttransformer_b200.models.native.model import build_model
    from nexttransformer_b200.native.optimizer import build_optimizer, set_schedule
    from nexttransformer_b200.runtime import checkpoint as ckpt
    from nexttransformer_b200.runtime.files import atomic_json
    from nexttransformer_b200.runtime.process import initialize, shutdown, synchronize
    from nexttransformer_b200.runtime.tracking import start_tracker
    seed = tc.seed if args.seed is None else args.seed
    rank, world, device = initialize(seed)
    out = args.output or Path(args.runtime_dir) / "runs" / (args.run_name or f"native_{args.config.stem}_seed{seed}")
    if rank == 0:
        out.mkdir(parents=True, exist_ok=True)
    accum = tc.accumulation(mc, world, micro)
    tok = load_tokenizer(args) if args.data == "bestfit" else None
    stream = make_stream(args, mc, rank, world, seed, tok)
    if args.data == "bestfit" and args.prefetch > 0:
        from nexttransformer_b200.runtime.prefetch import PrefetchStream
        stream = PrefetchStream(stream, args.prefetch)
    tasks = None
    if args.core is not None and tok is not None:
        from nexttransformer_b200.training.evals import load_core_bundle
        tasks = load_core_bundle(args.core)
    model = build_model(mc, device, seed=seed)
    # The dense model trains through the fused sm_100a path on CUDA; the optimizer then writes the
    # bf16 shadows that path reads.
    shadows = None
    if device.type == "cuda" and mc.architecture == "dense" and model.fused_supported():
        shadows = {p: s for p, s in model.fused_state().casts}
        model.use_fused = True
    optimizer = build_optimizer(model, tc, shadows=shadows)
    state = dict(step=0, input_tokens=0, training_seconds=0.0, smoke=bool(args.smoke_steps))
    if args.resume == "auto":
        if rank == 0:
            ckpt.set_aside_incomplete(out)
        done = ckpt.complete_checkpoints(out)
        if done:
            state = ckpt.load_checkpoint(out / f"checkpoint_{done[-1]:08d}", model, optimizer, stream, rank,
                                         world)["state"]
            if shadows is not None:
                model.refresh_shadows()
    stop = min(args.smoke_steps or tc.steps, tc.steps)
    every = args.checkpoint_every or tc.checkpoint_every
    phase = None
    with start_tracker(out, rank, args.wandb_mode, dict(model=asdict(mc), train=asdict(tc)), device) as tracker:
        model.train()
        if state["step"] == 0 and not args.smoke_steps:
            for event in scheduled_evaluations(args, model, tc, tok, tasks, 0, False, micro, rank, world, device):
                if rank == 0:
                    tracker.log(event)
        for step in range(state["step"], stop):
            model.set_circle_step(step + args.circle_stage_step)
            mult = set_schedule(optimizer, step, tc)
            synchronize(device)
            t0 = time.time()
            values = update(model, optimizer, stream, mc, tc, accum, micro, world, device,
                            step + args.circle_stage_step)
            if values is None:
                if rank == 0:
                    tracker.log({"event": "nonfinite", "step": step + 1})
                phase = "nonfinite"
                break
            synchronize(device)
            dt = time.time() - t0
            state.update(step=step + 1, input_tokens=state["input_tokens"] + int(values[4]),
                         training_seconds=state["training_seconds"] + dt)
            if rank == 0 and ((step + 1) % args.log_every == 0 or step + 1 == stop):
                R = mc.routing_steps
                tracker.log({"event": "train", "step": step + 1, "lm_loss": values[0], "router_loss": values[1],
                             "loss": values[6 + R], "objective": values[9 + R], "training_flops": values[2],
                             "active_depth_mean": values[5] / values[4],
                             "active_fraction": [v / values[4] for v in values[6:6 + R]],
                             "lr_multiplier": mult, "step_seconds": dt, "tokens_per_second": values[4] / dt,
                             "circle_stage": model.circle_stage() if mc.architecture == "circle" else None})
            if args.smoke_val_tokens and step + 1 == stop:
                from nexttransformer_b200.evaluation.bpb import evaluate_stream_loss
                res = evaluate_stream_loss(_LossView(model), mc, args.smoke_val_tokens, micro, rank, world, device,
                                           seed)
                if rank == 0:
                    tracker.log({"event": "validation", "step": step + 1, **res})
            if not args.smoke_steps or args.smoke_val_tokens:
                for event in scheduled_evaluations(args, model, tc, tok, tasks, step + 1, step + 1 == tc.steps, micro,
                                                   rank, world, device):
                    if rank == 0:
                        tracker.log(event)
            if (every and (step + 1) % every == 0) or step + 1 == stop:
                ckpt.save_checkpoint(out, model, optimizer, stream, mc, tc, state, rank, world)
        if rank == 0:
            atomic_json(out / "run_status.json", {"phase": phase or ("smoke" if args.smoke_steps else "complete"),
                                                  **state})
    shutdown()
    if phase == "nonfinite":
        sys.exit(NONFINITE_EXIT)
    return state


class _LossView(torch.nn.Module):
    """Adapts the native model to the ``model(x, y, loss_reduction='none')`` evaluation call."""

    def __init__(self, model):
        super().__init__()
        self.model = model

    def forward(self, x, y, loss_reduction="none"):
        return self.model(x, y, loss_reduction=loss_reduction)


if __name__ == "__main__":
    main()
