"""Trainer control flow on CPU: segments + resume are bitwise identical to a continuous run; two
gloo ranks train identical replicas; a non-finite loss stops the run with exit code 3."""
import json
import os

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import free_port

ARGS = ["--method", "gdn_hybrid", "--debug-scale", "--global-batch", "96", "--total-tokens", "960",
        "--micro-batch", "2", "--rolling-every", "2", "--rolling-keep", "3", "--val-every", "3", "--val-tokens", "48"]


def _params(out):
    from nexttransformer_b200.runtime.checkpoint import complete_checkpoints
    last = complete_checkpoints(out)[-1]
    return torch.load(out / f"checkpoint_{last:08d}" / "model.pt", weights_only=False)["model"]


def test_segments_resume_bitwise(tmp_path, monkeypatch):
    from nexttransformer_b200 import train
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    full = tmp_path / "full"
    train.main([*ARGS, "--output", str(full), "--steps", "5"])
    seg = tmp_path / "seg"
    train.main([*ARGS, "--output", str(seg), "--steps", "3"])
    train.main([*ARGS, "--output", str(seg), "--steps", "5", "--resume", "auto"])
    a, b = _params(full), _params(seg)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    events = [json.loads(l) for l in (seg / "metrics.jsonl").read_text().splitlines()]
    assert [e["step"] for e in events if e["event"] == "train"] == [1, 2, 3, 4, 5]
    assert any(e["event"] == "validation" for e in events)


def _rank(rank, world, port, out, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank), CUDA_VISIBLE_DEVICES="")
    from nexttransformer_b200 import train
    train.main([*ARGS, "--output", str(out), "--steps", "2"])
    q.put(rank)


def test_two_gloo_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, tmp_path, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert sorted(q.get() for _ in range(2)) == [0, 1]
    status = json.loads((tmp_path / "run_status.json").read_text())
    assert status["step"] == 2 and status["input_tokens"] == 192


def test_nonfinite_exit(tmp_path, monkeypatch):
    from nexttransformer_b200 import train
    from nexttransformer_b200.models import lm
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    orig = lm.LanguageModel.forward

    def poisoned(self, *a, **k):
        out = orig(self, *a, **k)
        return out * float("nan")
    monkeypatch.setattr(lm.LanguageModel, "forward", poisoned)
    with pytest.raises(SystemExit) as e:
        train.main([*ARGS, "--output", str(tmp_path), "--steps", "2"])
    assert e.value.code == train.NONFINITE_EXIT
    events = [json.loads(l) for l in (tmp_path / "metrics.jsonl").read_text().splitlines()]
    assert events[-1]["event"] == "nonfinite"


def test_run_records_schedule_budget_and_status(tmp_path, monkeypatch):
    """Validation follows --val-every, every update logs a device-free step time and grad norm, and
    the run ends with budget.json and run_status.json."""
    from nexttransformer_b200 import train
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    out = tmp_path / "run"
    train.main([*ARGS, "--output", str(out), "--steps", "4"])
    events = [json.loads(l) for l in (out / "metrics.jsonl").read_text().splitlines()]
    assert [e["step"] for e in events if e["event"] == "validation"] == [3, 4]
    steps = [e for e in events if e["event"] == "train"]
    assert all(e["grad_norm"] > 0 and e["step_seconds"] > 0 for e in steps)
    budget = json.loads((out / "budget.json").read_text())
    status = json.loads((out / "run_status.json").read_text())
    assert budget["step"] == 4 and status["step"] == 4 and status["phase"] == "stopped"
    assert (out / "val_00000003.json").exists()


def test_grad_norm_matches_direct_sum():
    from nexttransformer_b200.train import grad_norm_sq
    ps = [torch.nn.Parameter(torch.randn(5, 3)), torch.nn.Parameter(torch.randn(7)),
          torch.nn.Parameter(torch.randn(2, 2, dtype=torch.float64))]
    for p in ps:
        p.grad = torch.randn_like(p)
    want = sum(float(p.grad.double().square().sum()) for p in ps)
    assert abs(float(grad_norm_sq(ps)) - want) < 1e-5 * want     # fp32 norms per tensor
