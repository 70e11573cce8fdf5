"""Training entry point: ``python -m nexttransformer_b200.train`` (one process per GPU under torchrun).

Modes (reference: ``nexttransformer/train.py``):
  * ``--formal``: the configuration file must carry an admitted cost proof; every update is
    charged its audited cost in the ``BudgetState`` ledger; data layout, batch and schedule are
    the frozen protocol's.
  * ``--research`` (default): any configuration (file, ``--method`` candidate or debug scale),
    findings recorded in provenance; results are never admitted.
Per update: schedule -> micro-batches (forward/backward; fused sm_100a path on CUDA) ->
gradient norm (one multi-tensor norm) and the loss sums reduced over the ranks in ONE collective,
read by the host once -> non-finite check -> Muon/AdamW step (gradients reduced to their owners)
-> router-bias update -> budget charge and rolling cost-window check (``budget_anomaly``) ->
events (``metrics.jsonl``; step time from CUDA events, maximum over ranks) -> scheduled
evaluation (validation bits per byte on the protocol's schedule, CORE at the protocol's core
steps) -> checkpoints.  A completed run ends with the final train / validation bits per byte,
the final CORE score, ``budget.json`` and ``run_status.json`` with the budget's final status.
Resume: ``--resume auto`` restarts from the newest complete checkpoint (incomplete ones are moved
aside, later events archived); ``--max-wall-hours`` ends a segment after a checkpoint; a
non-finite loss or gradient records an event and exits with code 3.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
from dataclasses import asdict, replace
import json
import math
import os
from pathlib import Path
import sys
import time

import torch
import torch.distributed as dist

NONFINITE_EXIT = 3


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    mode = p.add_mutually_exclusive_group()
    mode.add_argument("--formal", action="store_true")
    mode.add_argument("--research", action="store_true")
    p.add_argument("--config", type=Path, help="configuration JSON (configs/<family>/<method>.json)")
    p.add_argument("--method", help="candidate configuration of a registered method (research mode)")
    p.add_argument("--debug-scale", action="store_true", help="tiny debug configuration of --method")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--data", choices=("bestfit", "synthetic"), default="synthetic")
    p.add_argument("--prefetch", type=int, default=2,
                   help="micro-batches packed ahead on a background thread (real data; 0: pack inline)")
    p.add_argument("--steps", type=int, default=0, help="stop after this update (0: protocol length)")
    p.add_argument("--total-tokens", type=int, default=0, help="research: token budget of the schedule")
    p.add_argument("--global-batch", type=int, default=0, help="research: tokens per update")
    p.add_argument("--resume", default="never", help="never | auto")
    p.add_argument("--max-wall-hours", type=float, default=0.)
    p.add_argument("--checkpoint-every", type=int, default=0, help="protocol checkpoints (permanent)")
    p.add_argument("--rolling-every", type=int, default=500)
    p.add_argument("--rolling-keep", type=int, default=2)
    p.add_argument("--val-every", type=int, default=0, help="research: validation cadence (0: protocol)")
    p.add_argument("--val-tokens", type=int, default=0)
    p.add_argument("--sparse-backend", choices=("reference", "kernel"), default="reference")
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--core", type=Path, help="CORE bundle (tasks.json + <label>.jsonl) scored at the core steps")
    p.add_argument("--tokenizer", type=Path, help="tokenizer directory (default: <resources>/tokenizer)")
    p.add_argument("--core-max-per-task", type=int, default=-1)
    p.add_argument("--deterministic-attention", action="store_true",
                   help="attention backward without atomics (dQ accumulated per query tile in a fixed order)")
    p.add_argument("--seed", type=int, default=42)
    args = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(args)
    if not args.formal:
        args.research = True
    if args.resume not in ("never", "auto"):
        p.error("--resume takes never or auto")
    if args.config is None and args.method is None:
        p.error("give --config or --method")
    if not hasattr(args, "core_max_tokens"):
        args.core_max_tokens = None
    return args


def grad_norm_sq(params):
    """Squared global gradient norm: one multi-tensor norm over the gradients (no copies)."""
    from nexttransformer_b200.optim.muon_adamw import grad_of
    grads = [g for g in (grad_of(p) for p in params) if g is not None]
    if not grads:
        return torch.zeros((), dtype=torch.float64)
    by_dtype = {}
    for g in grads:
        by_dtype.setdefault((g.device, g.dtype), []).append(g)
    total = None
    for group in by_dtype.values():
        norms = torch._foreach_norm(group)
        part = torch.stack([n.double() for n in norms]).square().sum()
        total = part if total is None else total + part
    return total


def load_model_config(args):
    from nexttransformer_b200.models.config import candidate_config, debug_config
    from nexttransformer_b200.protocol.admission import admit_config, review_config
    from nexttransformer_b200.protocol.spec import load_config
    findings, proof = [], None
    if args.config is not None:
        if args.formal:
            config, proof = admit_config(args.config)
        else:
            try:
                config, proof, findings = review_config(args.config)
            except (ValueError, KeyError, FileNotFoundError) as e:
                config, findings = load_config(args.config), [f"no usable cost proof: {e}"]
    else:
        if args.formal:
            raise ValueError("formal runs need an admitted configuration file")
        config = debug_config(args.method) if args.debug_scale else candidate_config(args.method)
        findings = ["candidate configuration without a cost proof"]
    return config, proof, findings


def _dense_anchor(args):
    """The dense FLOPs-per-token anchor of the configuration's cost evidence (None without one)."""
    if not getattr(args, "config", None):
        return None
    return json.loads(Path(args.config).read_text()).get("calibration", {}).get("dense_flops_per_token")


def stage_cost(proof, step):
    """Audited cost charged to update `step` (the stage that trains it)."""
    if proof is None:
        return None
    start = 0
    for s in proof["stages"]:
        if step < start + s["optimizer_steps"]:
            return s["cost"]["total"]
        start += s["optimizer_steps"]
    raise ValueError("update outside the audited stages")


def main(argv=None):
    args = parse(argv)
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.optim.groups import TrainConfig, protocol_groups, set_schedule
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW, grad_of
    from nexttransformer_b200.protocol.admission import BudgetState, data_layout, events_at
    from nexttransformer_b200.protocol.spec import Protocol
    from nexttransformer_b200.runtime import checkpoint as ckpt
    from nexttransformer_b200.runtime.data import SyntheticStream
    from nexttransformer_b200.runtime.files import atomic_json
    from nexttransformer_b200.runtime.process import initialize, reduce_max, reduce_sum, shutdown, synchronize
    from nexttransformer_b200.runtime.tracking import start_tracker

    proto = Protocol()
    config, proof, findings = load_model_config(args)
    rank, world, device = initialize(args.seed)
    out = Path(args.output)
    if rank == 0:
        out.mkdir(parents=True, exist_ok=True)
    if world > 1:
        dist.barrier()
    train = proto.train_config()
    if args.research and (args.total_tokens or args.global_batch):
        gb = args.global_batch or train.global_batch_tokens
        train = replace(train, global_batch_tokens=gb, total_tokens=args.total_tokens or gb * max(args.steps, 1))
    T = config.sequence_len
    micro = args.micro_batch or max(1, min(16, train.global_batch_tokens // (world * T)))
    if train.global_batch_tokens % (world * micro * T):
        raise ValueError("global batch must be divisible by world x micro batch x sequence")
    accum = train.global_batch_tokens // (world * micro * T)
    stream_rank, stream_world, shares = data_layout(rank, world)
    if args.data == "synthetic":
        stream = SyntheticStream(config.vocab_size, T, stream_rank, stream_world, seed=args.seed)
    else:
        from nexttransformer_b200.runtime.data import BestFitStream
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tok = BPETokenizer.from_directory(Path(args.resources) / "tokenizer")
        stream = BestFitStream(args.data_dir or Path(args.resources) / "base_data_climbmix", tok, "train",
                               stream_rank, stream_world, T)
        if args.prefetch > 0:
            from nexttransformer_b200.runtime.prefetch import PrefetchStream
            stream = PrefetchStream(stream, args.prefetch)

    model = build_model(config, device, seed=args.seed)
    model.set_sparse_backend(args.sparse_backend)
    stage = model.set_training_stage(0)
    shadows = {}
    if device.type == "cuda":    # every eligible projection on the sm_100a GEMM engine
        shadows = {p: s for p, s in model.fused_state().casts}
    optimizer = MuonAdamW(protocol_groups(model, train), shadows=shadows)
    budget = BudgetState()
    state = dict(step=0, input_tokens=0, training_seconds=0.0, budget=budget.state_dict(), findings=findings,
                 mode="formal" if args.formal else "research")
    if args.resume == "auto":
        if rank == 0:
            ckpt.set_aside_incomplete(out)
        if world > 1:
            dist.barrier()
        steps = ckpt.complete_checkpoints(out)
        if steps:
            saved = ckpt.load_checkpoint(out / f"checkpoint_{steps[-1]:08d}", model, optimizer, stream, rank, world)
            state = saved["state"]
            budget = BudgetState.from_state_dict(state["budget"])
            if rank == 0:
                from nexttransformer_b200.runtime.process import append_event
                _rewind_events(out, state["step"])
    if rank == 0:
        atomic_json(out / ("provenance.json" if state["step"] == 0 else f"resume_{state['step']:08d}.json"), dict(
            model=config.serialized(), train=asdict(train), world_size=world, micro_batch=micro,
            gradient_accumulation=accum, findings=findings, mode=state["mode"], torch=torch.__version__,
            dense_flops_per_token=_dense_anchor(args),
            device=torch.cuda.get_device_name(device) if device.type == "cuda" else "cpu", argv=sys.argv))
    stop = min(args.steps or train.steps, train.steps)
    val_every = args.val_every or proto.val_every
    started = time.time()
    phase = None
    dense_anchor = _dense_anchor(args)
    if args.deterministic_attention:
        from nexttransformer_b200.ops import attention as attention_ops
        attention_ops.set_deterministic(True)
    evaluator = _evaluator(args, model, config, train, rank, world, device, micro, stream_rank, stream_world)
    window = []
    start_ev = torch.cuda.Event(enable_timing=True) if device.type == "cuda" else None
    end_ev = torch.cuda.Event(enable_timing=True) if device.type == "cuda" else None
    with start_tracker(out, rank, args.wandb_mode, dict(model=config.serialized()), device) as tracker:
        model.train()

        def event(payload):
            if rank == 0:
                tracker.log(payload)

        def scheduled_evaluations(step):
            """Validation and CORE due after update ``step`` (formal: the protocol's schedule)."""
            if args.formal:
                due = events_at(step)
                due_val = due["val"] and step not in budget.val_steps
                due_core = due["core"] and not due["final"] and step not in budget.core_steps
            else:
                due_val = bool(args.val_tokens or args.data == "bestfit") and (step % val_every == 0 or step == stop)
                due_core = evaluator.has_core and step in proto.core_steps and step < proto.steps
            if due_val:
                result = evaluator.validation(args.val_tokens or proto.val_tokens)
                if args.formal:
                    budget.record_eval("val")
                payload = {"event": "validation", "step": step, **result}
                if "bpb" in result:
                    payload["val_bpb"] = result["bpb"]
                event(payload)
                if rank == 0:
                    atomic_json(out / f"val_{step:08d}.json", payload)
            if due_core and evaluator.has_core:
                result = evaluator.core()
                if args.formal:
                    budget.record_eval("core")
                payload = {"event": "core", "step": step, **result}
                event(payload)
                if rank == 0:
                    atomic_json(out / f"core_{step:08d}.json", payload)

        for step in range(state["step"], stop):
            if config.method == "ouro":
                stage = model.set_training_stage(step)
            model.set_step(step)
            mult = set_schedule(optimizer, step, train)
            synchronize(device)
            t0 = time.time()
            if start_ev is not None:
                start_ev.record()
            for p in model.parameters():
                p.grad = None
            if hasattr(model, "zero_main_grads"):
                model.zero_main_grads()
            totals = torch.zeros(5, device=device, dtype=torch.float64)  # lm, aux, tokens, |g|^2, non-finite
            for micro_i in range(accum):
                x, y = stream.batch(micro, device)
                if hasattr(model, "set_row_offset"):
                    model.set_row_offset(stream.rows - micro)
                loss = model(x, y)
                (loss / accum).backward()
                lm = model.last_lm_loss if model.last_lm_loss is not None else loss.detach()
                totals[:3] += torch.stack((lm.detach().double(), (loss.detach() - lm.detach()).double(),
                                           torch.full((), float(y.numel()), device=device, dtype=torch.float64)))
            gsq = grad_norm_sq(model.parameters()).to(device)
            totals[3] = gsq
            totals[4] = (~torch.isfinite(gsq) | ~torch.isfinite(totals[:2]).all()).double()
            reduce_sum(totals)            # one collective and one host read per update
            lm_sum, aux_sum, tokens, gsq_all, bad = totals.tolist()
            if bad:
                if rank == 0:
                    tracker.log({"event": "nonfinite", "step": step + 1, "lm_loss": lm_sum / (world * accum)})
                phase = "nonfinite"
                break
            optimizer.step()
            if hasattr(model, "update_router_bias"):
                model.update_router_bias()
            if end_ev is not None:
                end_ev.record()
            synchronize(device)
            dt = time.time() - t0
            if start_ev is not None:
                dt_dev = torch.tensor([start_ev.elapsed_time(end_ev) / 1e3], device=device, dtype=torch.float64)
                reduce_max(dt_dev)
                dt = float(dt_dev.item())
            tokens = int(tokens)
            if tokens != train.global_batch_tokens:
                raise RuntimeError("training input-token budget drift")
            cost = stage_cost(proof, step)
            if args.formal:
                budget.advance(tokens, cost)
            state.update(step=step + 1, input_tokens=state["input_tokens"] + tokens,
                         training_seconds=state["training_seconds"] + dt, budget=budget.state_dict())
            if cost is not None and dense_anchor:
                window = (window + [cost])[-proto.val_every:]
                rolling = sum(window) / (len(window) * proto.global_batch_tokens * dense_anchor) - 1
                if len(window) == proto.val_every and abs(rolling) > proto.routing_warning:
                    event({"event": "budget_anomaly", "step": step + 1, "rolling_relative_error": rolling})
            if rank == 0 and ((step + 1) % args.log_every == 0 or step + 1 == stop):
                tracker.log({"event": "train", "step": step + 1, "input_tokens": state["input_tokens"],
                             "lm_loss": lm_sum / (world * accum), "aux_loss": aux_sum / (world * accum),
                             "grad_norm": math.sqrt(gsq_all) if world == 1 else None,
                             "grad_norm_rank_sum_sq": gsq_all, "lr_multiplier": mult,
                             "stage": stage, "step_seconds": dt, "tokens_per_second": tokens / dt,
                             "theory_flops": cost})
            done = step + 1 == stop
            scheduled_evaluations(step + 1)
            wall_up = args.max_wall_hours and (time.time() - started) / 3600 >= args.max_wall_hours
            protocol_ckpt = args.checkpoint_every and (step + 1) % args.checkpoint_every == 0
            rolling_ckpt = args.rolling_every and (step + 1) % args.rolling_every == 0
            if protocol_ckpt or rolling_ckpt or done or wall_up:
                optimizer.flush()
                ckpt.save_checkpoint(out, model, optimizer, stream, config, train, state, rank, world)
                if rank == 0 and args.rolling_keep:
                    keep = {s for s in ckpt.complete_checkpoints(out)
                            if args.checkpoint_every and s % args.checkpoint_every == 0}
                    ckpt.prune_rolling(out, args.rolling_keep, protected=keep | {step + 1})
            if wall_up and not done:
                phase = "segment_end"
                break
        complete = phase is None and state["step"] == proto.steps
        if complete:
            # the final checkpoint precedes these evaluations; a resumed segment re-runs only them
            final = evaluator.final(proto.final_bpb_tokens)
            if rank == 0:
                atomic_json(out / "bpb_final.json", final)
            event({"event": "final_bpb", "step": proto.steps, "train": final["train"], "val": final["val"]})
            if evaluator.has_core and (not args.formal or proto.steps not in budget.core_steps):
                result = evaluator.core(final=True)
                if args.formal:
                    budget.record_eval("core")
                if rank == 0:
                    atomic_json(out / "core_final.json", {"step": proto.steps, **result})
                event({"event": "core", "step": proto.steps, **result})
        if rank == 0:
            budget_state = budget.state_dict()
            atomic_json(out / "budget.json", {"step": state["step"], **budget_state,
                                              "dense_flops_per_token": dense_anchor})
            final_status = budget.final_status(dense_anchor) if args.formal and dense_anchor else None
            atomic_json(out / "run_status.json", {
                "phase": phase or ("training_complete" if complete else "stopped"), "final_status": final_status,
                "evaluation_seconds": evaluator.seconds, **state})
    shutdown()
    if phase == "nonfinite":
        sys.exit(NONFINITE_EXIT)
    return state


def _evaluator(args, model, config, train, rank, world, device, micro, stream_rank, stream_world):
    """The run's evaluator: real-data bits per byte with ``--data bestfit``, CORE with ``--core``."""
    from nexttransformer_b200.training.evals import RunEvaluator, load_core_bundle
    tokenizer = tasks = None
    data_dir = None
    if args.data == "bestfit" or args.core:
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tokenizer = BPETokenizer.from_directory(args.tokenizer or Path(args.resources) / "tokenizer")
        data_dir = args.data_dir or Path(args.resources) / "base_data_climbmix"
    if args.core:
        tasks = load_core_bundle(args.core)
    return RunEvaluator(model, config, rank=rank, world=world, device=device, micro=micro, data=args.data,
                        data_dir=data_dir, tokenizer=tokenizer, core_tasks=tasks,
                        core_max_tokens=args.core_max_tokens, core_max_per_task=args.core_max_per_task,
                        seed=args.seed, stream_rank=stream_rank, stream_world=stream_world)


def _rewind_events(out, step):
    """Archive events past the resumed checkpoint so one active history remains."""
    metrics = Path(out) / "metrics.jsonl"
    if not metrics.exists():
        return
    keep, later = [], []
    for line in metrics.read_text().splitlines():
        try:
            ev = json.loads(line)
        except json.JSONDecodeError:
            later.append(line)
            continue
        (keep if ev.get("step", 0) <= step else later).append(line)
    if later:
        arch = Path(out) / "replayed_events" / str(time.time_ns())
        arch.mkdir(parents=True, exist_ok=True)
        (arch / "metrics.jsonl").write_text("\n".join(later) + "\n")
        tmp = metrics.with_suffix(".jsonl.tmp")
        tmp.write_text("\n".join(keep) + ("\n" if keep else ""))
        tmp.replace(metrics)


if __name__ == "__main__":
    main()
