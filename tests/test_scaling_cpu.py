"""Scaling-stage configuration, MoE recipe, per-node checkpoints and trainer on CPU (tiny shapes;
two gloo ranks stand for two nodes without a shared filesystem)."""
from dataclasses import replace
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nexttransformer_b200.scaling.config import (ScalingModelConfig, ScalingTrainConfig, config_hash, load_config,
                                                 write_config)

TINY = dict(width=48, heads=2, mlp_width=192, vocab_size=96, sequence_len=16, dense_layers=3, window_pattern="SL")


def _config(tmp_path, **train):
    kw = dict(total_tokens=128, global_batch_tokens=32, val_tokens=32, final_bpb_tokens=32, val_every=2,
              checkpoint_every=1, milestone_every=2, core_every=0)
    kw.update(train)
    path = tmp_path / "tiny.json"
    write_config(path, ScalingModelConfig(**TINY), ScalingTrainConfig(**kw))
    return path


def test_config_defaults_hash_and_rules(tmp_path):
    mc, tc = ScalingModelConfig(), ScalingTrainConfig()
    # the serialized form leaves the value-embedding switch out at its default
    assert "value_embeddings" not in mc.serialized()
    assert config_hash(mc, tc).startswith("f8f69c5183c9")
    assert tc.batch_scale == 2.0 and tc.is_milestone(10_000) and not tc.is_milestone(9_000)
    assert tc.core_steps()[-1] == tc.steps
    with pytest.raises(ValueError):
        ScalingTrainConfig(milestone_every=1500)
    with pytest.raises(ValueError):
        ScalingTrainConfig(total_tokens=3 * 2_097_152 + 1)
    path = _config(tmp_path)
    mc2, tc2 = load_config(path)
    assert mc2.width == 48 and tc2.steps == 4
    raw = json.loads(path.read_text())
    raw["train"]["global_batch_tokens"] = 40
    raw["train"]["total_tokens"] = 160
    (tmp_path / "bad.json").write_text(json.dumps(raw))
    with pytest.raises(ValueError):
        load_config(tmp_path / "bad.json")


def test_shipped_scaling_configs_load():
    root = os.path.join(os.path.dirname(__file__), "..", "configs", "scaling")
    for name in ("dense_200b.json", "t3_dense_l20.json", "t3_dense_l28.json"):
        mc, tc = load_config(os.path.join(root, name))
        assert mc.architecture == "dense" and tc.steps > 0


def test_moe_recipe_matches_manifest(tmp_path):
    from nexttransformer_b200.scaling.moe_recipe import MANIFEST, MoERecipe, load_t3_recipe
    data = json.loads(MANIFEST.read_text())
    for cell in data["cells"]:
        if cell["family"] in ("moe", "looped"):
            r = load_t3_recipe(cell["id"])
            assert r.estimate()["estimated_updates"] == cell["estimatedUpdates"], cell["id"]
    r = load_t3_recipe("moe-T3-L20")
    c = r.counts()
    assert r.expert_width == r.width // 4 and c["model_total"] == c["block_total"] + c["embedding_and_head"] + \
        c["native_small_parameters"]
    assert r.block_active() < c["block_total"]
    assert load_t3_recipe("kda-dsa-T3-L20").estimate()["estimated_updates"] is None
    dbg = r.debug()
    assert dbg.width == 32 and dbg.layers == 3
    with pytest.raises(ValueError):
        MoERecipe(layers=4, width=64, heads=4, expert_width=8)
    data["families"][1]["recipe"]["routedExperts"] = 128
    changed = tmp_path / "t3.json"
    changed.write_text(json.dumps(data))
    with pytest.raises(ValueError):
        load_t3_recipe("moe-T3-L20", changed)


def _final_weights(output, step, node=0):
    return torch.load(output / f"checkpoint_{step:08d}" / f"node_{node:03d}" / "model.pt", weights_only=False)["model"]


def test_scaling_smoke_resume_stop_and_benchmark(tmp_path, monkeypatch, capsys):
    from nexttransformer_b200.scaling import train
    monkeypatch.setenv("WORLD_SIZE", "1")
    cfg = _config(tmp_path)
    base = ["--config", str(cfg), "--micro-batch", "1", "--log-every", "1"]
    full = train.main(base + ["--output", str(tmp_path / "full"), "--smoke-steps", "3"])
    assert full["step"] == 3 and full["input_tokens"] == 96
    status = json.loads((tmp_path / "full" / "run_status.json").read_text())
    assert status["phase"] == "smoke_complete"
    assert (tmp_path / "full" / "checkpoint_00000003" / "node_000" / "complete.json").exists()
    # a second launch into the same output without --resume is refused
    with pytest.raises(ValueError):
        train.main(base + ["--output", str(tmp_path / "full"), "--smoke-steps", "3"])
    # stop after one update, resume for the rest: the same weights as the continuous run
    seg = tmp_path / "seg"
    got = train.main(base + ["--output", str(seg), "--smoke-steps", "3", "--stop-after", "1"])
    assert got["step"] == 1
    assert json.loads((seg / "run_status.json").read_text())["phase"] == "stopped"
    # an incomplete newer checkpoint is set aside, never deleted
    (seg / "checkpoint_00000002" / "node_000").mkdir(parents=True)
    train.main(base + ["--output", str(seg), "--smoke-steps", "3", "--resume", "auto"])
    assert list((seg / "abandoned").rglob("checkpoint_00000002"))
    a, b = _final_weights(tmp_path / "full", 3), _final_weights(seg, 3)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    # a STOP file stops after the current update and is consumed
    stop = tmp_path / "stop"
    stop.mkdir()
    (stop / "STOP").write_text("")
    got = train.main(base + ["--output", str(stop), "--smoke-steps", "3"])
    assert got["step"] == 1 and (stop / "STOP.consumed-00000001").exists()
    # benchmark mode writes no checkpoint and prints one summary line
    capsys.readouterr()
    train.main(["--config", str(cfg), "--micro-batch", "1", "--benchmark", "2", "--output", str(tmp_path / "bench")])
    summary = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert summary["event"] == "benchmark" and summary["measured_steps"] == 1
    assert not list((tmp_path / "bench").glob("checkpoint_*"))


def test_scaling_nonfinite_exits_3(tmp_path, monkeypatch):
    from nexttransformer_b200.scaling import train
    monkeypatch.setenv("WORLD_SIZE", "1")
    cfg = _config(tmp_path)
    from nexttransformer_b200.models.native import model as native_model
    real = native_model.NativeExperiment.forward

    def poisoned(self, *a, **k):
        out = real(self, *a, **k)
        if isinstance(out, dict):
            out["loss"] = out["loss"] * float("nan")
        return out
    monkeypatch.setattr(native_model.NativeExperiment, "forward", poisoned)
    with pytest.raises(SystemExit) as e:
        train.main(["--config", str(cfg), "--micro-batch", "1", "--output", str(tmp_path / "nan"), "--smoke-steps", "2"])
    assert e.value.code == train.NONFINITE_EXIT


def test_dry_run(tmp_path, capsys):
    from nexttransformer_b200.scaling import train
    train.main(["--config", str(_config(tmp_path)), "--dry-run", "--world-size", "2", "--micro-batch", "1"])
    out = json.loads(capsys.readouterr().out)
    assert out["accumulation"] == 1 and out["scaling_parameters"] > 0 and out["muon_weight_decay"] > 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_nodes(rank, port, cfg, output, argv_extra, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="2", RANK=str(rank),
                      LOCAL_RANK="0", LOCAL_WORLD_SIZE="1")
    from nexttransformer_b200.scaling import train
    try:
        state = train.main(["--config", cfg, "--micro-batch", "1", "--output", output] + argv_extra)
        results[rank] = state["step"]
    except Exception as e:  # reported to the parent
        results[rank] = repr(e)


@pytest.mark.timeout(300)
def test_two_nodes_checkpoint_and_resume(tmp_path):
    cfg = str(_config(tmp_path, global_batch_tokens=32, total_tokens=128))
    out = tmp_path / "run"
    with mp.Manager() as manager:
        for extra in (["--smoke-steps", "2", "--stop-after", "1"], ["--smoke-steps", "2", "--resume", "auto", "--bf16-grad-reduce"]):
            results = manager.dict()
            port = _port()
            mp.start_processes(_two_nodes, args=(port, cfg, str(out), extra, results), nprocs=2, start_method="spawn")
            assert dict(results) == {0: results[0], 1: results[1]}
            assert all(isinstance(v, int) for v in results.values()), dict(results)
    # each node wrote its own complete checkpoint of the same model
    for node in (0, 1):
        assert (out / "checkpoint_00000002" / f"node_{node:03d}" / "complete.json").exists()
    a, b = _final_weights(out, 2, 0), _final_weights(out, 2, 1)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert (out / "status.node000.json").exists() and (out / "status.node001.json").exists()


def test_routed_ffn_oracle_matches_moe_layer():
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.moe import MoEFFN
    from nexttransformer_b200.scaling.reference_blocks import RoutedFFN
    cfg = debug_config("dsa")
    torch.manual_seed(0)
    oracle = RoutedFFN(cfg, 8, 2, cfg.width // 4)
    layer = MoEFFN(cfg.width, 8, 2, cfg.width // 4, shared=1)
    layer.load_state_dict({**oracle.state_dict(), "expert_bias": torch.zeros(8)}, strict=False)
    x = torch.randn(2, 8, cfg.width)
    got = layer(x)
    got = got[0] if isinstance(got, tuple) else got
    torch.testing.assert_close(got, oracle(x), rtol=1e-5, atol=1e-5)


def test_kda_dsa_group_and_rule():
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.scaling.reference_blocks import KdaDsaGroup, RoutedFFN, rotary, shared_expert_rule
    cfg = debug_config("dsa")
    rule = shared_expert_rule(cfg, 8, 2, cfg.width // 4)
    assert not isinstance(rule(0), RoutedFFN) and isinstance(rule(1), RoutedFFN)
    group = KdaDsaGroup(cfg, rule)
    x = torch.randn(2, cfg.sequence_len, cfg.width)
    for step in (0, cfg.burnin_steps):
        group.zero_grad(set_to_none=True)
        out, aux = group(x, rotary(cfg), step)
        (out.square().mean() + aux).backward()
        assert torch.isfinite(out).all()


def test_recompute_layers_give_the_same_update(tmp_path, monkeypatch):
    from nexttransformer_b200.scaling import train
    monkeypatch.setenv("WORLD_SIZE", "1")
    cfg = _config(tmp_path)
    base = ["--config", str(cfg), "--micro-batch", "1", "--smoke-steps", "1"]
    train.main(base + ["--output", str(tmp_path / "plain")])
    train.main(base + ["--output", str(tmp_path / "recompute"), "--recompute-layers", "-1"])
    a, b = _final_weights(tmp_path / "plain", 1), _final_weights(tmp_path / "recompute", 1)
    for k in a:
        torch.testing.assert_close(a[k], b[k], rtol=0, atol=1e-6)


def test_complete_run_exports_a_record(tmp_path, monkeypatch):
    from nexttransformer_b200.scaling import export, train
    monkeypatch.setenv("WORLD_SIZE", "1")
    cfg = _config(tmp_path)
    state = train.main(["--config", str(cfg), "--micro-batch", "1", "--output", str(tmp_path / "run")])
    assert state["step"] == 4
    assert json.loads((tmp_path / "run" / "run_status.json").read_text())["phase"] == "training_complete"
    rec = export.record(tmp_path / "run", cfg, "tiny", "Tiny", "dense")
    assert [v["step"] for v in rec["val"]] == [0, 2, 4] and rec["finalVal"] == rec["finalVal"]
    results = tmp_path / "results"
    export.write(results, rec)
    export.write(results, rec)                     # identical export: no-op
    assert export.check(results) == []
    changed = dict(rec, name="Other")
    with pytest.raises(ValueError):
        export.write(results, changed)
    # a smoke run is never exported
    train.main(["--config", str(cfg), "--micro-batch", "1", "--output", str(tmp_path / "smoke"), "--smoke-steps", "4"])
    with pytest.raises(ValueError):
        export.record(tmp_path / "smoke", cfg, "tiny", "Tiny", "dense")


def test_core_evaluation_at_core_steps(tmp_path, monkeypatch):
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    from nexttransformer_b200.scaling import train
    monkeypatch.setenv("WORLD_SIZE", "1")
    docs = ["the quick brown fox jumps over the lazy dog %d" % i for i in range(50)]
    tok = BPETokenizer.train_from_iterator(docs, vocab_size=300)
    tok.save(tmp_path / "tok")
    cfg = tmp_path / "core.json"
    write_config(cfg, ScalingModelConfig(**dict(TINY, vocab_size=320)),
                 ScalingTrainConfig(total_tokens=64, global_batch_tokens=32, val_tokens=32, final_bpb_tokens=32,
                                    val_every=2, checkpoint_every=1, milestone_every=2, core_every=1))
    bundle = tmp_path / "bundle"
    bundle.mkdir()
    (bundle / "tasks.json").write_text(json.dumps([{"label": "lm", "random_baseline": 0.0,
                                                    "meta": {"task_type": "language_modeling", "num_fewshot": 0}}]))
    (bundle / "lm.jsonl").write_text("".join(json.dumps({"context": "the quick brown", "continuation": " fox"}) + "\n"
                                             for _ in range(3)))
    train.main(["--config", str(cfg), "--micro-batch", "1", "--output", str(tmp_path / "run"), "--core", str(bundle),
                "--tokenizer", str(tmp_path / "tok")])
    events = [json.loads(l) for l in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    core = [e for e in events if e["event"] == "core"]
    assert [e["step"] for e in core] == [1, 2]
    assert core[0]["coreContext"]["truncation"] == "none" and 0 <= core[-1]["core_metric"] <= 1
    assert (tmp_path / "run" / "core_00000001.json").exists() and (tmp_path / "run" / "core_final.json").exists()


def test_real_data_validation_is_bpb(tmp_path, monkeypatch):
    import pyarrow as pa
    import pyarrow.parquet as pq
    from nexttransformer_b200.runtime.files import VALIDATION_SHARD
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    from nexttransformer_b200.scaling import export, train
    monkeypatch.setenv("WORLD_SIZE", "1")
    docs = ["the quick brown fox jumps over the lazy dog %d" % i for i in range(300)]
    data = tmp_path / "data"
    data.mkdir()
    pq.write_table(pa.table({"text": docs}), data / "shard_00000.parquet")
    pq.write_table(pa.table({"text": docs[:60]}), data / VALIDATION_SHARD)
    BPETokenizer.train_from_iterator(docs, vocab_size=300).save(tmp_path / "res" / "tokenizer")
    cfg = tmp_path / "bpb.json"
    write_config(cfg, ScalingModelConfig(**dict(TINY, vocab_size=320)),
                 ScalingTrainConfig(total_tokens=64, global_batch_tokens=32, val_tokens=32, final_bpb_tokens=32,
                                    val_every=1, checkpoint_every=1, milestone_every=2, core_every=0))
    train.main(["--config", str(cfg), "--micro-batch", "1", "--output", str(tmp_path / "run"), "--data", "bestfit",
                "--resources", str(tmp_path / "res"), "--data-dir", str(data)])
    events = [json.loads(l) for l in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    val = [e for e in events if e["event"] == "validation"]
    assert [e["step"] for e in val] == [0, 1, 2] and all(0 < e["val_bpb"] < 100 for e in val)
    rec = export.record(tmp_path / "run", cfg, "bpb", "BPB", "dense")
    assert rec["metric"] == "val_bpb" and len(rec["val"]) == 3


@pytest.mark.parametrize("burnin", [True, False])
def test_kda_dsa_group_is_causal_and_trains_its_indexer(burnin):
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.scaling.reference_blocks import KdaDsaGroup, rotary
    torch.manual_seed(42)
    cfg = debug_config("dsa")
    group = KdaDsaGroup(cfg)
    assert [m.kind for m in group.mixers] == ["kda", "kda", "kda", "dsa"]
    x = torch.randn(1, cfg.sequence_len, cfg.width)
    step = cfg.burnin_steps - int(burnin)
    out, aux = group(x, rotary(cfg), step)
    assert group.mixers[-1].in_burnin is burnin
    (out.square().mean() + aux).backward()
    grad = group.mixers[-1].index_q.weight.grad
    assert torch.isfinite(grad).all() and grad.abs().sum() > 0
    changed = x.clone()
    changed[:, -2:] += torch.randn_like(changed[:, -2:])
    with torch.no_grad():
        changed_out, _ = group(changed, rotary(cfg), step)
    torch.testing.assert_close(out[:, :-2], changed_out[:, :-2])
