"""One gym job in its own process: cost inspection or a research training run of a candidate.

    python -m nexttransformer_b200.gym.worker JOB.json

The job file names the candidate's plugin directory, the profile and the work; the parent sets
``NEXTTRANSFORMER_METHOD_PATHS`` to that directory (so the registry discovers the plugin before
any model code is imported), ``CUDA_VISIBLE_DEVICES`` to the leased GPUs, and a scrubbed
environment.  Progress goes to ``progress.json`` after every update and the outcome to
``result.json`` next to the job file; the exit code is 0 on success.

Training: the candidate is built at the profile's shell dimensions, trains ``target_update``
updates of ``rows`` synthetic rows (iid uniform tokens; research runs never read the validation
data) with AdamW through ``ResearchDP`` over the visible GPUs (or the CPU), and reports the loss
curve, tokens per second and the FLOPs charged (audited FLOPs per token x tokens trained).
"""
import json
import sys
import time
from dataclasses import replace
from pathlib import Path


def profile_config(method, profile):
    from nexttransformer_b200.models.config import candidate_config
    c = candidate_config(method)
    return replace(c, scale="custom", width=profile["width"], heads=profile["heads"], layers=profile["layers"],
                   mlp_width=profile["mlp_width"], vocab_size=profile["vocab_size"],
                   sequence_len=profile["sequence_len"])


def cost(method, profile):
    import torch
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.protocol.compute import flops_per_token
    cfg = profile_config(method, profile)
    with torch.device("meta"):
        model = build_model(cfg, "meta", seed=0)
    params = sum(p.numel() for p in model.parameters())
    fpt = flops_per_token(cfg, batch=min(profile["rows"], 8))
    return dict(parameters=int(params), flops_per_token=float(fpt),
                flops_per_update=float(fpt) * profile["rows"] * profile["sequence_len"])


def train(job, out):
    import torch
    from nexttransformer_b200.gym.research import ResearchDP
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.runtime.data import SyntheticStream
    profile = job["profile"]
    cfg = profile_config(job["method"], profile)
    devices = [f"cuda:{i}" for i in range(torch.cuda.device_count())] or ["cpu"]
    model = build_model(cfg, devices[0], seed=job.get("seed", 0))
    dp = ResearchDP(model, devices, lambda m: torch.optim.AdamW(m.parameters(), lr=job.get("lr", 3e-4)))
    stream = SyntheticStream(cfg.vocab_size, cfg.sequence_len, seed=job.get("seed", 0))

    def loss_fn(m, x, y):
        return m(x, y)
    losses, t0 = [], time.time()
    tokens = 0
    for step in range(job["target_update"]):
        x, y = stream.cpu_batch(profile["rows"])
        losses.append(dp.step(x, y, profile["micro_rows"], loss_fn))
        tokens += x.numel()
        (out / "progress.json").write_text(json.dumps(dict(update=step + 1, loss=losses[-1], tokens=tokens)))
    seconds = time.time() - t0
    fpt = cost(job["method"], profile)["flops_per_token"]
    return dict(losses=losses, tokens=tokens, seconds=seconds, tokens_per_second=tokens / max(seconds, 1e-9),
                devices=devices, flops=fpt * tokens)


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    job_path = Path(argv[0])
    job = json.loads(job_path.read_text())
    out = job_path.parent
    try:
        result = cost(job["method"], job["profile"]) if job["kind"] == "cost" else train(job, out)
        (out / "result.json").write_text(json.dumps(dict(ok=True, **result)))
        return 0
    except Exception as e:  # reported to the service as the job's failure
        (out / "result.json").write_text(json.dumps(dict(ok=False, error=f"{type(e).__name__}: {e}")))
        return 1


if __name__ == "__main__":
    raise SystemExit(main())
