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


def test_native_full_run_scheduled_evaluations(tmp_path, monkeypatch):
    """A full (non-smoke) run on real data logs counted validation BPB at every validation step,
    CORE at the final step and the final train / validation BPB."""
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from nexttransformer_b200.native import train
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    monkeypatch.setenv("WORLD_SIZE", "1")
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta"]
    docs = [" ".join(words[(i + j) % 6] for j in range(3 + i % 11)) for i in range(300)]
    data = tmp_path / "data"
    data.mkdir()
    for k, name in enumerate(("shard_00000.parquet", "shard_06542.parquet")):
        pq.write_table(pa.table({"text": docs[k * 150:(k + 1) * 150]}), data / name, row_group_size=25)
    BPETokenizer.train_from_iterator(docs, vocab_size=300).save(tmp_path / "res" / "tokenizer")
    bundle = tmp_path / "bundle"
    bundle.mkdir()
    (bundle / "tasks.json").write_text(json.dumps([{"label": "lm", "random_baseline": 0.0,
                                                    "meta": {"task_type": "language_modeling", "num_fewshot": 0}}]))
    (bundle / "lm.jsonl").write_text(json.dumps({"context": "alpha beta", "continuation": " gamma"}) + "\n")
    cfg = tmp_path / "mor.json"
    write_config(cfg, NativeModelConfig(**dict(TINY, architecture="mor", vocab_size=320)),
                 NativeTrainConfig(total_tokens=64, global_batch_tokens=32, val_tokens=32, final_bpb_tokens=32,
                                   val_every=1, checkpoint_every=2))
    state = train.main(["--config", str(cfg), "--output", str(tmp_path / "run"), "--micro-batch", "1",
                        "--data", "bestfit", "--data-dir", str(data), "--resources", str(tmp_path / "res"),
                        "--core", str(bundle)])
    assert state["step"] == 2
    events = [json.loads(l) for l in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    val = [e for e in events if e["event"] == "validation"]
    assert [e["step"] for e in val] == [0, 1, 2] and all(e["input_tokens"] == 32 and e["val_bpb"] > 0 for e in val)
    assert "mean_recursions" in val[0]
    core = [e for e in events if e["event"] == "core"]
    assert [e["step"] for e in core] == [2] and core[0]["full_core"]
    final = [e for e in events if e["event"] == "final_bpb"]
    assert len(final) == 1 and final[0]["train_bpb"] > 0 and final[0]["val_bpb"] > 0
