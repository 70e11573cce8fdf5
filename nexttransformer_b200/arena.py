"""Research arena: disclosure cards and the scope of an arena or method pull request.

    python -m nexttransformer_b200.arena --check [--results DIR]
    python -m nexttransformer_b200.arena --scope BASE

``--check`` validates every card ``<results>/arena/<id>.json``: the disclosure schema (sections and
their keys), the vocabularies (status, involvement level, verification, selection signals), dates
and the base commit, the counts, and for admitted / complete entries the model card, the run
records and the admitted configuration they name.  ``--scope BASE`` classifies the files changed
since the merge base with BASE when a card is among them or a method plugin is added, and fails when
such a change touches the training contract, the evaluation, another method's model or frozen
evidence.  Neither imports torch.

The card format, its vocabularies and the scope categories are those of the reference
(``nexttransformer/arena.py:1-218``), so cards written for one validate under the other; the
checks here are a rule table of their own and the protected paths are this package's.
"""
import argparse
import json
import re
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
RESULTS = REPO / "results"
PACKAGE = "nexttransformer_b200/"

VERSION = "arena-v1"
TRAINING_PROTOCOL = "nextt-reference-50b-v1"
LEVELS = ("L0", "L1", "L2", "L3")
STATUSES = ("admitted", "complete", "legacy", "retracted")
VERIFICATION = ("self-reported", "reproduced", "maintainer")
SIGNALS = ("train-loss", "dev-bpb", "validation-bpb", "core", "other")
RESERVED_SIGNALS = ("validation-bpb", "core")   # the formal run's metrics never select candidates
SCHEMA = {
    None: ("id", "name", "methodId", "runIds", "arenaProtocol", "status", "statusNote", "submitted",
           "verification", "researcher", "research", "novelty", "artifacts"),
    "researcher": ("people", "llms", "framework", "involvement", "involvementNote"),
    "research": ("start", "end", "baseCommit", "candidatesTrained", "formalAttempts", "formalNote", "gpuHours",
                 "hardware", "computeNote", "internet", "selectionSignal"),
    "novelty": ("closestPrior", "statement"),
    "artifacts": ("checkpointUrl", "logsUrl", "traceUrl", "historyUrl", "codeUrl"),
}
_DATE = re.compile(r"\d{4}-\d{2}-\d{2}")
_COMMIT = re.compile(r"[0-9a-f]{7,40}")

# Scope of a pull request: the first rule whose prefix matches decides.
DOCS = "docs/"
CONTRACT = tuple(PACKAGE + p for p in (
    "models/shell.py", "models/lm.py", "models/fused_dense.py", "protocol/", "evaluation/", "runtime/", "training/",
    "checks/", "native/", "csrc/", "ops/", "optim/", "parallel/", "__init__.py", "arena.py", "audit_run.py",
    "train.py", "evaluate.py", "prepare.py", "generate.py", "inference.py")) + (
    "bench.py", "__graft_entry__.py", "launch/", ".github/", "pytest.ini")
FROZEN = ("results/runs/", "evidence/")


def _count(v):
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


def _people_ok(c):
    return isinstance(c["researcher"]["people"], list) and all(p.get("name") and p.get("role")
                                                               for p in c["researcher"]["people"])


def _llms_ok(c):
    llms = c["researcher"]["llms"]
    return isinstance(llms, list) and bool(llms) and all(m.get("name") and "version" in m and m.get("role")
                                                         for m in llms)


def _signals(c):
    s = c["research"]["selectionSignal"]
    return s if isinstance(s, list) else []


def _final(c):
    return c["status"] in ("admitted", "complete")


# (predicate, message); each runs on a card whose schema is complete
CARD_RULES = (
    (lambda c: c["arenaProtocol"] == VERSION, f"arenaProtocol is not {VERSION}"),
    (lambda c: c["status"] in STATUSES, f"status must be one of {STATUSES}"),
    (lambda c: _final(c) or bool(c["statusNote"]), "a legacy or retracted entry needs statusNote"),
    (lambda c: c["verification"] in VERIFICATION, f"verification must be one of {VERIFICATION}"),
    (lambda c: isinstance(c["runIds"], list), "runIds must be a list"),
    (lambda c: c["researcher"]["involvement"] in LEVELS, f"involvement must be one of {LEVELS}"),
    (lambda c: bool(c["researcher"]["involvementNote"]), "involvementNote is empty"),
    (_people_ok, "every person needs a name and a role"),
    (_llms_ok, "researcher.llms needs at least one LLM with name, version and role"),
    (lambda c: isinstance(c["researcher"]["framework"], dict) and bool(c["researcher"]["framework"].get("name")),
     "researcher.framework needs a name ('none' if none)"),
    (lambda c: all(_DATE.fullmatch(str(d)) for d in (c["submitted"], c["research"]["start"], c["research"]["end"])),
     "dates must be YYYY-MM-DD"),
    (lambda c: bool(_COMMIT.fullmatch(str(c["research"]["baseCommit"]))), "baseCommit must be a commit hash"),
    (lambda c: _count(c["research"]["candidatesTrained"]) and _count(c["research"]["formalAttempts"]),
     "candidatesTrained and formalAttempts must be counts"),
    (lambda c: c["research"]["gpuHours"] is None or (isinstance(c["research"]["gpuHours"], (int, float))
                                                     and not isinstance(c["research"]["gpuHours"], bool)
                                                     and c["research"]["gpuHours"] >= 0),
     "gpuHours must be a non-negative number or null"),
    (lambda c: isinstance(c["research"]["internet"], bool), "research.internet must be true or false"),
    (lambda c: bool(_signals(c)) and set(_signals(c)) <= set(SIGNALS), f"selectionSignal must list values of {SIGNALS}"),
    (lambda c: not _final(c) or not set(_signals(c)) & set(RESERVED_SIGNALS),
     "validation BPB and CORE belong to the formal run and cannot select candidates"),
    (lambda c: isinstance(c["novelty"]["closestPrior"], list) and bool(c["novelty"]["statement"]),
     "novelty needs closestPrior and a statement"),
    (lambda c: all(str(v).startswith("https://") for v in c["artifacts"].values() if v is not None),
     "artifact links must be HTTPS"),
    (lambda c: c["status"] != "complete" or bool(c["runIds"]), "a complete entry names its run"),
    (lambda c: c["status"] != "complete" or bool(c["artifacts"]["checkpointUrl"] and c["artifacts"]["logsUrl"]),
     "a complete entry links its final checkpoint and training logs"),
)


def card_problems(card, name):
    """Problems of one card on its own (schema first: the rules run only on a complete schema)."""
    problems = []
    for section, keys in SCHEMA.items():
        part = card if section is None else card.get(section)
        if not isinstance(part, dict):
            problems.append(f"{name}: missing {section}")
            continue
        missing = [k for k in keys if k not in part]
        if missing:
            problems.append(f"{name}: {section or 'card'} missing {missing}")
    if problems:
        return problems
    return [f"{name}: {msg}" for rule, msg in CARD_RULES if not rule(card)]


def _load_dir(path):
    return [json.loads(p.read_text()) for p in sorted(Path(path).glob("*.json"))]


def check(root=RESULTS, registered=None, config_of=None):
    """Problems of every card under ``root/arena`` and the records each names.

    ``registered``: method names of the registry (default: ``models.registry``); ``config_of(method)``
    returns the admitted configuration's path (default: ``protocol.spec.config_path``)."""
    root = Path(root)
    if registered is None:
        from nexttransformer_b200.models.registry import FAMILY
        registered = set(FAMILY)
    if config_of is None:
        from nexttransformer_b200.protocol.spec import config_path as config_of
    model_cards = {c["id"] for c in _load_dir(root / "methods")}
    runs = {r["id"]: r for r in _load_dir(root / "runs")}
    problems, entered = [], set()
    for path in sorted((root / "arena").glob("*.json")):
        name = f"arena/{path.name}"
        try:
            card = json.loads(path.read_text())
        except json.JSONDecodeError as e:
            problems.append(f"{name}: {e}")
            continue
        if card.get("id") != path.stem:
            problems.append(f"{name}: id differs from the file name")
        if card.get("methodId") in entered:
            problems.append(f"{name}: another card already enters {card.get('methodId')}")
        entered.add(card.get("methodId"))
        own = card_problems(card, name)
        problems += own
        if own:
            continue
        method = card["methodId"]
        if method not in model_cards:
            problems.append(f"{name}: no model card methods/{method}.json")
        named = []
        for rid in card["runIds"]:
            run = runs.get(rid)
            if run is None:
                problems.append(f"{name}: no run record {rid}")
            elif run.get("methodId") != method:
                problems.append(f"{name}: run {rid} belongs to {run.get('methodId')}")
            else:
                named.append(run)
        if not _final(card):
            continue
        if method not in registered:
            problems.append(f"{name}: {method} is not a registered method")
            continue
        cfg = Path(config_of(method))
        if not cfg.exists():
            problems.append(f"{name}: no admitted configuration {cfg.name}")
            continue
        admitted = json.loads(cfg.read_text()).get("model_hash")
        if card["status"] == "complete":
            for run in named:
                if (run.get("protocol"), run.get("status"), run.get("complete"), run.get("reportedAudit")) != \
                        (TRAINING_PROTOCOL, "finished", True, "matched"):
                    problems.append(f"{name}: run {run['id']} is not a complete, matched {TRAINING_PROTOCOL} run")
                if (run.get("proof") or {}).get("model_hash") != admitted:
                    problems.append(f"{name}: run {run['id']} was not trained from the admitted configuration")
    return problems


def is_card(path):
    return re.fullmatch(r"results/arena/[^/]+\.json", path) is not None


def _config_verdict(kind, path, base_text, repo):
    if kind == "A":
        return "ok", "new configuration"
    if kind == "D":
        return "blocked", "configurations are never deleted"
    before = json.loads(base_text(path) or "{}")
    after = json.loads((Path(repo) / path).read_text())
    same = all(before.get(k) == after.get(k) for k in ("model", "model_hash", "protocol_hash"))
    return ("ok", "calibration refresh; model unchanged") if same else ("blocked", "changes another method's model")


def _by_kind(kind, table, default):
    return table.get(kind, default)


def classify(changes, base_text=lambda path: None, repo=REPO):
    """(verdict, status, path, reason) for each ``git diff --name-status`` row; verdict is ``ok``,
    ``review`` or ``blocked``."""
    out = []
    for status, path in changes:
        kind = status[0]
        if path.startswith(CONTRACT):
            v = ("blocked", "fixed by the training contract or the arena")
        elif is_card(path):
            v = ("blocked", "cards are never deleted") if kind == "D" else ("ok", "disclosure card")
        elif path.startswith(FROZEN):
            v = ("ok", "new record or evidence") if kind == "A" else ("blocked", "published records and evidence are frozen")
        elif path.startswith("results/methods/"):
            v = _by_kind(kind, {"A": ("ok", "new model card"), "D": ("blocked", "model cards are never deleted")},
                         ("review", "changes an existing model card"))
        elif path.startswith("configs/"):
            v = _config_verdict(kind, path, base_text, repo)
        elif path.startswith(PACKAGE + "methods/"):
            v = _by_kind(kind, {"A": ("ok", "new plugin file"), "D": ("blocked", "plugins are never deleted")},
                         ("review", "changes an existing plugin"))
        elif path.startswith((PACKAGE + "models/", "tests/")):
            v = ("ok", "new file") if kind == "A" else ("review", "changes shared code or tests")
        elif path.startswith(DOCS):
            v = ("ok", "documentation")
        else:
            v = ("review", "outside the arena surface")
        out.append((v[0], status, path, v[1]))
    return out


def adds_method(changes):
    """True when the changes add a method plugin (a new ``methods/<name>/method.json``)."""
    return any(s[0] == "A" and p.startswith(PACKAGE + "methods/") and p.endswith("/method.json") for s, p in changes)


def scope(base, repo=REPO):
    """Classified changes since the merge base with ``base``; None when no card changed and no
    plugin was added."""
    def git(*args):
        return subprocess.run(["git", *args], cwd=repo, capture_output=True, text=True, check=True).stdout
    mb = git("merge-base", base, "HEAD").strip()
    rows = [tuple(line.split("\t", 1)) for line in git("diff", "--name-status", "--no-renames", mb, "HEAD").splitlines()]
    if not any(is_card(p) for _, p in rows) and not adds_method(rows):
        return None

    def at_base(path):
        try:
            return git("show", f"{mb}:{path}")
        except subprocess.CalledProcessError:
            return None
    return classify(rows, at_base, repo)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    act = p.add_mutually_exclusive_group(required=True)
    act.add_argument("--check", action="store_true", help="validate every card under <results>/arena/")
    act.add_argument("--scope", metavar="BASE", help="classify the files a pull request changes since BASE")
    p.add_argument("--results", type=Path, default=RESULTS)
    a = p.parse_args(argv)
    if a.check:
        problems = check(a.results)
        n = len(list((a.results / "arena").glob("*.json")))
        print("\n".join(problems) if problems else f"{n} arena cards are valid")
        return 1 if problems else 0
    rows = scope(a.scope)
    if rows is None:
        print("No disclosure card changed and no method plugin added; nothing to classify.")
        return 0
    for verdict, status, path, reason in rows:
        print(f"{verdict:8} {status:2} {path}  ({reason})")
    return 1 if any(r[0] == "blocked" for r in rows) else 0


if __name__ == "__main__":
    raise SystemExit(main())
