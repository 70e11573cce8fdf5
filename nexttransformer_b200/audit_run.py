"""Read-only cumulative audit of a finished formal run directory, and its export as a results record
(``nexttransformer/audit_run.py`` and ``export_run.py`` of the reference, for the run directories
this package's trainer writes).

    python -m nexttransformer_b200.audit_run RUN_DIR --method gdn [--output audits/gdn.json]
    python -m nexttransformer_b200.audit_run RUN_DIR --method gdn --export results/gdn.json --name "Gated DeltaNet"
    python -m nexttransformer_b200.audit_run --check results/
    python -m nexttransformer_b200.audit_run RUN_DIR --frozen audits/gdn.json --export results/gdn.json

The audit re-reads everything the trainer wrote and checks it against the protocol: the ledger in
``run_status.json`` (all updates and input tokens, the protocol fingerprint, the validation / CORE
schedule, cumulative FLOPs within the protocol's tolerance of tokens x the dense anchor), the
training events (strictly increasing steps, input tokens = step x global batch, finite losses), the
validation events against their ``val_*.json`` files, and the provenance of every segment
(identical model and training configuration, formal mode, a batch layout that fills the global
batch).  The report records scientific quantities and fingerprints only - no host names, paths,
devices or timings - and the command exits non-zero when a check fails.  An export refuses a run
whose audit failed; ``--check`` validates every record of a results directory.

``--frozen AUDIT`` exports an archived run under the accounting its audit was made with, without
re-auditing it under the current ledger (``nexttransformer/export_frozen.py`` of the reference):
the run's ``metrics.jsonl`` must still hash to the audit's digest, the audit must have passed, and
every field of the record must equal the audit's; the record carries the audit's own sha256.
"""
import argparse
from datetime import date
import hashlib
import json
import math
from pathlib import Path

from nexttransformer_b200.protocol.spec import Protocol

CHECKS = [
    "run_status.json: complete at the final update; ledger updates, input tokens and protocol fingerprint",
    "cumulative theory FLOPs within the protocol tolerance of input tokens x the dense anchor",
    "train events: strictly increasing steps, input_tokens == step x global batch, finite losses",
    "validation events equal to their val_*.json files",
    "every segment: identical model and training configuration, formal mode, registered batch layout",
]
RECORD_FIELDS = ("schema", "method", "name", "status", "step", "val", "protocol_hash", "audit")


def _val_metric(event):
    return event.get("val_bpb", event.get("val_loss"))


def audit(run, method, protocol=None, dense_flops_per_token=None):
    """(report, problems) for run directory `run`."""
    P = protocol or Protocol()
    run = Path(run)
    problems = []

    def need(ok, message):
        if not ok:
            problems.append(message)

    def load(name):
        return json.loads((run / name).read_text())

    status = load("run_status.json")
    ledger = status.get("budget", {})
    need(status.get("phase") == "complete" and status.get("step") == P.steps, "run_status: not complete at the final update")
    need(ledger.get("optimizer_step") == P.steps and ledger.get("input_tokens") == P.total_tokens,
         "ledger: updates or input tokens differ from the protocol")
    need(ledger.get("protocol_hash") == P.fingerprint, "ledger: protocol fingerprint differs")

    names = ["provenance.json", *sorted(f.name for f in run.glob("resume_*.json"))]
    first = load(names[0])
    anchor = dense_flops_per_token or first.get("dense_flops_per_token")
    cumulative = None
    if anchor:
        cumulative = ledger.get("theory_flops", 0) / (P.total_tokens * anchor) - 1
        need(abs(cumulative) <= P.cumulative_tolerance,
             f"cumulative FLOP error {cumulative:.4%} exceeds {P.cumulative_tolerance:.0%}")
    else:
        problems.append("no dense FLOP anchor to check the cumulative charge against")

    events = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines() if line.strip()]
    train = [e for e in events if e["event"] == "train"]
    steps = [e["step"] for e in train]
    need(bool(train) and steps[-1] == P.steps, "train: the last event is not the final update")
    need(all(a < b for a, b in zip(steps, steps[1:])), "train: steps are not strictly increasing")
    need(all(e["input_tokens"] == e["step"] * P.global_batch_tokens for e in train),
         "train: input_tokens != step x global batch")
    need(all(math.isfinite(e["lm_loss"]) for e in train), "train: non-finite loss")
    need(not any(e["event"] == "nonfinite" for e in events), "a non-finite update was recorded")

    val = [e for e in events if e["event"] == "validation"]
    by_step = {e["step"]: e for e in val}
    files = sorted(run.glob("val_*.json"))
    need(len(files) == len(val), f"validation: {len(files)} val_*.json files for {len(val)} events")
    for f in files:
        v = json.loads(f.read_text())
        need(_val_metric(by_step.get(v["step"], {})) == _val_metric(v), f"{f.name}: differs from metrics.jsonl")

    segments = []
    for name in names:
        p = load(name)
        need(p["model"] == first["model"] and p["train"] == first["train"], f"{name}: configuration differs")
        need(p.get("mode") == "formal", f"{name}: not a formal segment")
        need(p["world_size"] * p["micro_batch"] * p["gradient_accumulation"] * P.sequence_len == P.global_batch_tokens,
             f"{name}: batch layout does not fill the global batch")
        step = 0 if name == "provenance.json" else int(name[len("resume_"):-len(".json")])
        segments.append(dict(file=name, step=step, world=p["world_size"], micro=p["micro_batch"],
                             accumulation=p["gradient_accumulation"]))

    final_val = [e for e in val if e["step"] == P.steps]
    digest = hashlib.sha256((run / "metrics.jsonl").read_bytes()).hexdigest()
    report = dict(schema="run-audit-v1", method=method, date=date.today().isoformat(), checks=CHECKS,
                  ok=not problems, problems=problems, optimizer_steps=ledger.get("optimizer_step"),
                  input_tokens=ledger.get("input_tokens"), theory_flops=ledger.get("theory_flops"),
                  dense_flops_per_token=anchor, cumulative_relative_error=cumulative, train_events=len(train),
                  validation_events=len(val), last_loss=train[-1]["lm_loss"] if train else None,
                  final_val=_val_metric(final_val[0]) if final_val else None, segments=segments,
                  protocol_hash=P.fingerprint, model=first["model"], metrics_sha256=digest,
                  accounting=first.get("accounting", "ledger-v1"))
    return report, problems


def export_record(report, name):
    """A results record of an audited run; refuses a failed audit."""
    if not report["ok"]:
        raise ValueError("the run's audit failed: " + "; ".join(report["problems"]))
    return dict(schema="run-record-v1", method=report["method"], name=name, status="complete",
                step=report["optimizer_steps"], val=report["final_val"], protocol_hash=report["protocol_hash"],
                audit={k: report[k] for k in ("date", "cumulative_relative_error", "theory_flops", "segments")})


FROZEN_NOTE = "Frozen accounting: the record keeps the cumulative FLOPs and fingerprints of its original audit."


def export_frozen(run, audit_path, name=None):
    """Record of an archived run under its audit's (frozen) accounting; raises on any difference
    between the run directory, the audit and the record."""
    run, audit_path = Path(run), Path(audit_path)
    raw = audit_path.read_bytes()
    report = json.loads(raw)
    if hashlib.sha256((run / "metrics.jsonl").read_bytes()).hexdigest() != report.get("metrics_sha256"):
        raise ValueError("metrics.jsonl differs from the audited archive")
    events = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines() if line.strip()]
    train = [e for e in events if e["event"] == "train"]
    val = [e for e in events if e["event"] == "validation"]
    record = export_record(report, name or report["method"])
    observed = {"optimizer_steps": train[-1]["step"] if train else None, "train_events": len(train),
                "validation_events": len(val), "final_val": _val_metric(val[-1]) if val else None}
    mismatched = [k for k, v in observed.items() if report.get(k) != v]
    if mismatched or record["val"] != report["final_val"] or record["step"] != report["optimizer_steps"]:
        raise ValueError(f"archived run differs from its audit: {mismatched or ['record']}")
    record.update(accounting=report.get("accounting", "ledger-v1"), comparisonNote=FROZEN_NOTE,
                  auditSha256=hashlib.sha256(raw).hexdigest(), metrics_sha256=report["metrics_sha256"])
    return record


def check_records(directory, protocol=None):
    """Problems of every record in `directory` (required fields, protocol, finite values)."""
    P = protocol or Protocol()
    problems = []
    for path in sorted(Path(directory).glob("*.json")):
        record = json.loads(path.read_text())
        missing = [k for k in RECORD_FIELDS if k not in record]
        if missing:
            problems.append(f"{path.name}: missing {', '.join(missing)}")
            continue
        if record["protocol_hash"] != P.fingerprint:
            problems.append(f"{path.name}: another protocol")
        if record["step"] != P.steps or not (isinstance(record["val"], float) and math.isfinite(record["val"])):
            problems.append(f"{path.name}: incomplete run or non-finite validation")
    return problems


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("run_dir", type=Path, nargs="?")
    parser.add_argument("--method")
    parser.add_argument("--output", type=Path, help="audit report (default: audits/<method>.json)")
    parser.add_argument("--dense-flops-per-token", type=float, help="FLOP anchor (default: the provenance's)")
    parser.add_argument("--export", type=Path, help="also write the results record here")
    parser.add_argument("--name", help="display name of the exported record")
    parser.add_argument("--check", type=Path, help="validate every record of this results directory")
    parser.add_argument("--frozen", type=Path, help="export RUN_DIR under this archived audit's accounting")
    args = parser.parse_args(argv)
    if args.frozen:
        if args.run_dir is None or args.export is None:
            parser.error("--frozen needs RUN_DIR and --export")
        record = export_frozen(args.run_dir, args.frozen, args.name)
        if args.export.exists():
            if json.loads(args.export.read_text()) != record:
                raise SystemExit(f"{args.export}: published frozen record differs")
            print(f"unchanged {args.export}")
            return
        args.export.parent.mkdir(parents=True, exist_ok=True)
        args.export.write_text(json.dumps(record, indent=1) + "\n")
        print(f"wrote {args.export}")
        return
    if args.check:
        problems = check_records(args.check)
        for p in problems:
            print("  " + p)
        raise SystemExit(1 if problems else 0)
    if args.run_dir is None or not args.method:
        parser.error("an audit needs RUN_DIR and --method")
    report, problems = audit(args.run_dir, args.method, dense_flops_per_token=args.dense_flops_per_token)
    out = args.output or Path("audits") / f"{args.method}.json"
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(report, indent=1) + "\n")
    print(f"wrote {out}: {'all checks passed' if not problems else f'{len(problems)} problem(s)'}")
    for p in problems:
        print("  " + p)
    if args.export and not problems:
        record = export_record(report, args.name or args.method)
        if args.export.exists() and json.loads(args.export.read_text()) != record:
            raise SystemExit(f"{args.export} exists with another record; records are immutable")
        args.export.parent.mkdir(parents=True, exist_ok=True)
        args.export.write_text(json.dumps(record, indent=1) + "\n")
    raise SystemExit(1 if problems else 0)


if __name__ == "__main__":
    main()
