"""Export a finished scaling-stage run as a results record, or check every record
(``nexttransformer/scaling/export.py`` of the reference, for this package's scaling trainer).

    python -m nexttransformer_b200.scaling.export RUN_DIR --config configs/scaling/dense_200b.json \
        --id dense_200b --name "Dense, 200B tokens" --family dense [--results results/scaling]
    python -m nexttransformer_b200.scaling.export --check [--results results/scaling]

The export reads rank zero's records (provenance.json, run_status.json, metrics.jsonl, val_*.json,
bpb_final.json) and refuses a run unless training completed under this configuration (same
configuration hash, not a smoke run), every scheduled validation is present and equal to its file,
and the final evaluation agrees with the event history.  A record keeps scientific quantities only
(no host names, paths, devices or commands); records are immutable: an identical export is a no-op.
"""
import argparse
import json
import math
from pathlib import Path

from nexttransformer_b200.scaling.config import config_hash, load_config

FIELDS = ("id", "name", "family", "protocol", "configSha256", "model", "parameters", "training", "source", "val",
          "finalVal")


def _metric(event, prefix=""):
    """Validation value of an event: bits per byte with real data, the synthetic-stream loss otherwise."""
    for key in ("val_bpb", "val_loss"):
        if prefix + key in event:
            return event[prefix + key]
    raise ValueError("an evaluation record without a validation value")


def record(run, config, run_id, name, family):
    run = Path(run)
    mc, tc = load_config(config)
    provenance = json.loads((run / "provenance.json").read_text())
    status = json.loads((run / "run_status.json").read_text())
    events = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines() if line.strip()]
    if status.get("phase") != "training_complete" or status.get("step") != tc.steps or provenance.get("smoke"):
        raise ValueError("the run has not completed training")
    if provenance.get("config_sha256") != config_hash(mc, tc):
        raise ValueError("the run was trained under another configuration")
    val = {e["step"]: e for e in events if e["event"] == "validation"}
    if sorted(val) != tc.validation_steps():
        raise ValueError(f"validation events at {sorted(val)}, scheduled {tc.validation_steps()}")
    for step, e in val.items():
        saved = json.loads((run / f"val_{step:08d}.json").read_text())
        if _metric(saved) != _metric(e):
            raise ValueError(f"val_{step:08d}.json differs from the event history")
    finals = [e for e in events if e["event"] == "final_bpb"]
    final = json.loads((run / "bpb_final.json").read_text())
    if len(finals) != 1 or _metric(finals[0], "final_") != _metric(final["val"]):
        raise ValueError("the final evaluation is missing or differs from the event history")
    train = [e for e in events if e["event"] == "train"]
    if not train or not all(math.isfinite(e["lm_loss"]) for e in train):
        raise ValueError("missing or non-finite training losses")
    return {"id": run_id, "name": name, "family": family, "protocol": tc.protocol, "configSha256": config_hash(mc, tc),
            "model": mc.serialized(), "parameters": provenance["parameters"],
            "training": {"steps": tc.steps, "input_tokens": status["input_tokens"],
                         "global_batch_tokens": tc.global_batch_tokens, "world_size": provenance["world_size"],
                         "last_lm_loss": train[-1]["lm_loss"]},
            "source": provenance["source_sha256"],
            "metric": "val_bpb" if "val_bpb" in final["val"] else "val_loss",
            "val": [{"step": s, "value": _metric(val[s])} for s in sorted(val)],
            "finalVal": _metric(final["val"])}


def write(results, rec):
    path = Path(results) / f"{rec['id']}.json"
    if path.exists():
        if json.loads(path.read_text()) != json.loads(json.dumps(rec)):
            raise ValueError(f"{path} exists with another record; records are immutable")
        return path
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(rec, indent=1) + "\n")
    return path


def check(results):
    problems = []
    for path in sorted(Path(results).glob("*.json")):
        rec = json.loads(path.read_text())
        missing = [f for f in FIELDS if f not in rec]
        if missing:
            problems.append(f"{path.name}: missing {', '.join(missing)}")
        elif rec["id"] != path.stem or not math.isfinite(rec["finalVal"]):
            problems.append(f"{path.name}: id differs from the file name or the final value is not finite")
    return problems


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("run_dir", type=Path, nargs="?")
    p.add_argument("--config", type=Path)
    p.add_argument("--id")
    p.add_argument("--name")
    p.add_argument("--family")
    p.add_argument("--results", type=Path, default=Path("results/scaling"))
    p.add_argument("--check", action="store_true")
    a = p.parse_args(argv)
    if a.check:
        problems = check(a.results)
        for problem in problems:
            print("  " + problem)
        raise SystemExit(1 if problems else 0)
    if not (a.run_dir and a.config and a.id and a.name and a.family):
        p.error("an export needs RUN_DIR, --config, --id, --name and --family")
    print(write(a.results, record(a.run_dir, a.config, a.id, a.name, a.family)))


if __name__ == "__main__":
    main()
