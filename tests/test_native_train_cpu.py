"""Native-track trainer, benchmark and preflight on CPU (tiny configurations)."""
import json

import pytest
import torch

from nexttransformer_b200.models.native.config import NativeModelConfig, NativeTrainConfig, write_config

TINY = dict(width=48, heads=2, mlp_width=192, vocab_size=96, sequence_len=16, dense_layers=4, pre_layers=1,
            core_layers=2, post_layers=1, fourier_dim=8, window_pattern="SL")


def _config(tmp_path, arch):
    kw = dict(TINY, architecture=arch)
    if arch == "circle":
        kw.update(circle_max_steps=6, circle_target_steps=4.0, circle_random_warmup=1, circle_route_transition=2)
    path = tmp_path / f"{arch}.json"
    write_config(path, NativeModelConfig(**kw), NativeTrainConfig(total_tokens=64, global_batch_tokens=32,
                                                                  val_tokens=32, final_bpb_tokens=32, val_every=1,
                                                                  checkpoint_every=2))
    return path


@pytest.mark.parametrize("arch", ["dense", "mor", "loopformer", "circle"])
def test_native_smoke_and_resume(tmp_path, arch, monkeypatch):
    from nexttransformer_b200.native import train
    monkeypatch.setenv("WORLD_SIZE", "1")
    cfg = _config(tmp_path, arch)
    full = train.main(["--config", str(cfg), "--output", str(tmp_path / "full"), "--smoke-steps", "2",
                       "--micro-batch", "1", "--log-every", "1"])
    assert full["step"] == 2 and full["input_tokens"] == 64
    events = [json.loads(l) for l in (tmp_path / "full" / "metrics.jsonl").read_text().splitlines()]
    losses = [e["lm_loss"] for e in events if e["event"] == "train"]
    assert len(losses) == 2 and all(l == l for l in losses)
    # one update, checkpoint, resume for the second: same final weights as the continuous run
    train.main(["--config", str(cfg), "--output", str(tmp_path / "seg"), "--smoke-steps", "1", "--micro-batch", "1"])
    train.main(["--config", str(cfg), "--output", str(tmp_path / "seg"), "--smoke-steps", "2", "--micro-batch", "1",
                "--resume", "auto"])
    a = torch.load(tmp_path / "full" / "checkpoint_00000002" / "model.pt", weights_only=False)["model"]
    b = torch.load(tmp_path / "seg" / "checkpoint_00000002" / "model.pt", weights_only=False)["model"]
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_native_dry_run(tmp_path, capsys):
    from nexttransformer_b200.native import train
    cfg = _config(tmp_path, "mor")
    train.main(["--config", str(cfg), "--dry-run", "--world-size", "2", "--micro-batch", "1"])
    out = json.loads(capsys.readouterr().out)
    assert out["accumulation"] == 1 and out["parameters"] > 0 and out["train_GFLOPs_per_input_token"] > 0


def test_preflight_halves_on_oom(tmp_path):
    from nexttransformer_b200.native import preflight
    cfg = _config(tmp_path, "dense")
    calls = []

    def runner(cmd, log, timeout):
        batch = int(cmd[cmd.index("--micro-batch") + 1])
        calls.append(batch)
        result = cmd[cmd.index("--output") + 1]
        if batch > 1:
            open(log, "w").write("torch.OutOfMemoryError: CUDA out of memory")
            return 1
        open(log, "w").write("ok")
        open(result, "w").write(json.dumps({"tokens_per_second": 1.0}))
        return 0
    got = preflight.main(["--config", str(cfg), "--output", str(tmp_path / "pf.json"), "--micro-batch", "2",
                          "--gpus", "1"], runner=runner, busy="")
    assert got == 1 and calls == [2, 1]
    assert json.loads((tmp_path / "pf.json").read_text())["status"] == "passed"
    with pytest.raises(RuntimeError):
        preflight.main(["--config", str(cfg), "--output", str(tmp_path / "pf2.json")], runner=runner, busy="123")
