"""Run audit and export on a synthetic run directory of a tiny protocol."""
from dataclasses import replace
import json

import pytest

from nexttransformer_b200.audit_run import audit, check_records, export_record
from nexttransformer_b200.protocol.spec import Protocol

P = replace(Protocol(), total_tokens=4 * 4096, global_batch_tokens=4096, sequence_len=512, val_every=2,
            core_steps=(4,))
ANCHOR = 1000.0


def _run(tmp_path):
    run = tmp_path / "run"
    run.mkdir()
    ledger = dict(protocol_hash=P.fingerprint, optimizer_step=4, input_tokens=P.total_tokens,
                  theory_flops=int(P.total_tokens * ANCHOR * 1.005), val_steps=[0, 2, 4], core_steps=[4])
    (run / "run_status.json").write_text(json.dumps(dict(phase="complete", step=4, budget=ledger)))
    seg = dict(model={"method": "dense"}, train={"seed": 42}, world_size=8, micro_batch=1, gradient_accumulation=1,
               mode="formal")
    (run / "provenance.json").write_text(json.dumps(seg))
    (run / "resume_00000002.json").write_text(json.dumps(seg))
    events = [dict(event="validation", step=0, val_loss=5.0)]
    for s in range(1, 5):
        events.append(dict(event="train", step=s, input_tokens=s * 4096, lm_loss=5.0 - 0.1 * s))
        if s % 2 == 0:
            events.append(dict(event="validation", step=s, val_loss=5.0 - 0.1 * s))
    (run / "metrics.jsonl").write_text("".join(json.dumps(e) + "\n" for e in events))
    for e in events:
        if e["event"] == "validation":
            (run / f"val_{e['step']:08d}.json").write_text(json.dumps(e))
    return run


def test_audit_passes_and_exports(tmp_path):
    run = _run(tmp_path)
    report, problems = audit(run, "dense", protocol=P, dense_flops_per_token=ANCHOR)
    assert problems == [] and report["ok"] and len(report["segments"]) == 2
    assert abs(report["cumulative_relative_error"] - 0.005) < 1e-6
    record = export_record(report, "Dense")
    results = tmp_path / "results"
    results.mkdir()
    (results / "dense.json").write_text(json.dumps(record))
    assert check_records(results, protocol=P) == []
    (results / "broken.json").write_text(json.dumps({"method": "x"}))
    assert check_records(results, protocol=P)


def test_audit_finds_problems(tmp_path):
    run = _run(tmp_path)
    v = json.loads((run / "val_00000002.json").read_text())
    v["val_loss"] = 0.0
    (run / "val_00000002.json").write_text(json.dumps(v))
    seg = json.loads((run / "resume_00000002.json").read_text())
    seg["mode"] = "research"
    (run / "resume_00000002.json").write_text(json.dumps(seg))
    report, problems = audit(run, "dense", protocol=P, dense_flops_per_token=ANCHOR * 1.1)
    assert not report["ok"]
    text = " ".join(problems)
    assert "val_00000002.json" in text and "formal" in text and "cumulative" in text
    with pytest.raises(ValueError):
        export_record(report, "Dense")


def test_frozen_export_checks_the_archive(tmp_path):
    from nexttransformer_b200.audit_run import export_frozen
    run = _run(tmp_path)
    report, problems = audit(run, "dense", protocol=P, dense_flops_per_token=ANCHOR)
    assert not problems
    path = tmp_path / "audit.json"
    path.write_text(json.dumps(report))
    record = export_frozen(run, path, "Dense")
    assert record["val"] == report["final_val"] and record["metrics_sha256"] == report["metrics_sha256"]
    assert len(record["auditSha256"]) == 64 and record["accounting"] == "ledger-v1"
    with open(run / "metrics.jsonl", "a") as f:
        f.write(json.dumps(dict(event="train", step=5, input_tokens=5 * 4096, lm_loss=1.0)) + "\n")
    with pytest.raises(ValueError, match="archive"):
        export_frozen(run, path)
    bad = dict(report, ok=False, problems=["x"])
    path.write_text(json.dumps(bad))
    (tmp_path / "b").mkdir()
    run2 = _run(tmp_path / "b")
    bad["metrics_sha256"] = audit(run2, "dense", protocol=P, dense_flops_per_token=ANCHOR)[0]["metrics_sha256"]
    path.write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="audit failed"):
        export_frozen(run2, path)
