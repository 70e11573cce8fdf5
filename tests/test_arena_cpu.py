"""Arena disclosure cards and pull-request scope (arena.py)."""
import copy
import json
import subprocess

import pytest

from nexttransformer_b200 import arena


def _card(**over):
    card = {
        "id": "probe", "name": "Probe", "methodId": "probe", "runIds": ["probe-run"], "arenaProtocol": arena.VERSION,
        "status": "complete", "statusNote": "", "submitted": "2026-05-01", "verification": "self-reported",
        "researcher": {"people": [{"name": "A", "role": "lead"}], "llms": [{"name": "m", "version": "1", "role": "coder"}],
                       "framework": {"name": "none"}, "involvement": "L2", "involvementNote": "wrote the code"},
        "research": {"start": "2026-04-01", "end": "2026-04-20", "baseCommit": "abc1234", "candidatesTrained": 3,
                     "formalAttempts": 1, "formalNote": "", "gpuHours": 12.5, "hardware": "8xB200", "computeNote": "",
                     "internet": False, "selectionSignal": ["dev-bpb"]},
        "novelty": {"closestPrior": ["x"], "statement": "new"},
        "artifacts": {"checkpointUrl": "https://ckpt", "logsUrl": "https://logs", "traceUrl": None, "historyUrl": None,
                      "codeUrl": None},
    }
    for k, v in over.items():
        card[k] = v
    return card


@pytest.fixture
def results(tmp_path):
    root = tmp_path / "results"
    for d in ("arena", "methods", "runs"):
        (root / d).mkdir(parents=True)
    (root / "methods" / "probe.json").write_text(json.dumps({"id": "probe"}))
    (root / "runs" / "probe-run.json").write_text(json.dumps({
        "id": "probe-run", "methodId": "probe", "protocol": arena.TRAINING_PROTOCOL, "status": "finished",
        "complete": True, "reportedAudit": "matched", "proof": {"model_hash": "h1"}}))
    cfg = tmp_path / "probe.json"
    cfg.write_text(json.dumps({"model_hash": "h1"}))
    return root, dict(registered={"probe"}, config_of=lambda m: cfg)


def _write(root, card):
    (root / "arena" / f"{card['id']}.json").write_text(json.dumps(card))


def test_valid_complete_card(results):
    root, kw = results
    _write(root, _card())
    assert arena.check(root, **kw) == []


@pytest.mark.parametrize("edit,needle", [
    (lambda c: c["research"].update(selectionSignal=["core"]), "formal run"),
    (lambda c: c["research"].update(selectionSignal=["core"]) or c.update(status="legacy", statusNote="old"), None),
    (lambda c: c.update(status="legacy"), "statusNote"),
    (lambda c: c["researcher"].update(llms=[]), "llms"),
    (lambda c: c["research"].update(baseCommit="main"), "baseCommit"),
    (lambda c: c["research"].update(candidatesTrained=True), "counts"),
    (lambda c: c["artifacts"].update(traceUrl="http://x"), "HTTPS"),
    (lambda c: c["artifacts"].update(logsUrl=None), "training logs"),
    (lambda c: c.update(submitted="May 1"), "dates"),
    (lambda c: c["research"].pop("gpuHours"), "missing"),
])
def test_card_rules(results, edit, needle):
    root, kw = results
    card = copy.deepcopy(_card())
    edit(card)
    _write(root, card)
    problems = arena.check(root, **kw)
    if needle is None:
        assert problems == []
    else:
        assert problems and any(needle in p for p in problems), problems


def test_records_named_by_a_card(results):
    root, kw = results
    _write(root, _card(runIds=["missing"]))
    assert any("no run record" in p for p in arena.check(root, **kw))
    run = json.loads((root / "runs" / "probe-run.json").read_text())
    run["proof"]["model_hash"] = "other"
    (root / "runs" / "probe-run.json").write_text(json.dumps(run))
    _write(root, _card())
    assert any("admitted configuration" in p for p in arena.check(root, **kw))
    assert any("not a registered" in p for p in arena.check(root, registered=set(), config_of=kw["config_of"]))


def test_classify_scope():
    P = arena.PACKAGE
    rows = dict((p, v) for v, s, p, r in arena.classify([
        ("A", "results/arena/probe.json"), ("D", "results/arena/old.json"), ("M", P + "protocol/spec.py"),
        ("A", P + "methods/probe/method.json"), ("M", P + "methods/xsa/__init__.py"), ("A", "results/runs/r.json"),
        ("M", "results/runs/r.json"), ("A", "tests/test_probe.py"), ("M", "README.md")]))
    assert rows == {"results/arena/probe.json": "ok", "results/arena/old.json": "blocked",
                    P + "protocol/spec.py": "blocked", P + "methods/probe/method.json": "ok",
                    P + "methods/xsa/__init__.py": "review", "results/runs/r.json": "blocked",
                    "tests/test_probe.py": "ok", "README.md": "review"}


def test_scope_in_a_git_repository(tmp_path):
    def git(*a):
        subprocess.run(["git", *a], cwd=tmp_path, check=True, capture_output=True)
    git("init", "-q", "-b", "main")
    git("config", "user.email", "t@t")
    git("config", "user.name", "t")
    (tmp_path / "configs").mkdir()
    (tmp_path / "configs" / "m.json").write_text(json.dumps({"model": {"w": 1}, "model_hash": "a", "tokens": 1}))
    git("add", "-A")
    git("commit", "-qm", "base")
    git("checkout", "-qb", "entry")
    (tmp_path / "configs" / "m.json").write_text(json.dumps({"model": {"w": 1}, "model_hash": "a", "tokens": 2}))
    (tmp_path / "results" / "arena").mkdir(parents=True)
    (tmp_path / "results" / "arena" / "c.json").write_text("{}")
    git("add", "-A")
    git("commit", "-qm", "entry")
    rows = arena.scope("main", repo=tmp_path)
    verdicts = {p: v for v, s, p, r in rows}
    assert verdicts == {"configs/m.json": "ok", "results/arena/c.json": "ok"}
    (tmp_path / "configs" / "m.json").write_text(json.dumps({"model": {"w": 2}, "model_hash": "b"}))
    git("commit", "-qam", "change model")
    assert {p: v for v, s, p, r in arena.scope("main", repo=tmp_path)}["configs/m.json"] == "blocked"
