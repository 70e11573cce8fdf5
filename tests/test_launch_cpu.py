"""Launch scripts: the torchrun command line and the scaling watchdog's restart rules (fake node script)."""
import json
import os
from pathlib import Path
import subprocess

ROOT = Path(__file__).resolve().parents[1]


def test_train_sh_dry_run_and_layout_rule():
    env = dict(os.environ, DRY_RUN="1", NNODES="2", NPROC_PER_NODE="4", NODE_RANK="1", MASTER_ADDR="10.0.0.1")
    out = subprocess.run([str(ROOT / "launch/train.sh"), "--config", "c.json", "--formal"], env=env,
                         capture_output=True, text=True, check=True).stdout
    assert "--nnodes 2" in out and "--node-rank 1" in out and "nexttransformer_b200.train" in out
    env.update(NNODES="1", NPROC_PER_NODE="3")
    bad = subprocess.run([str(ROOT / "launch/train.sh"), "--config", "c.json"], env=env, capture_output=True)
    assert bad.returncode == 2
    ok = subprocess.run([str(ROOT / "launch/train.sh"), "--config", "c.json", "--smoke-steps", "2"], env=env,
                        capture_output=True)
    assert ok.returncode == 0


def _watchdog(tmp_path, phases):
    """Run the watchdog with a fake node script that writes the next phase (or none) per launch."""
    plan = tmp_path / "plan.json"
    plan.write_text(json.dumps(phases))
    fake = tmp_path / "node.sh"
    fake.write_text(f"""#!/usr/bin/env bash
python3 - <<'PY'
import json, pathlib
plan = pathlib.Path("{plan}")
phases = json.loads(plan.read_text())
phase = phases.pop(0)
plan.write_text(json.dumps(phases))
if phase:
    pathlib.Path("{tmp_path}/out/status.node000.json").write_text(json.dumps({{"phase": phase}}))
PY
exit 1
""")
    fake.chmod(0o755)
    (tmp_path / "out").mkdir(exist_ok=True)
    env = dict(os.environ, OUTPUT_DIR=str(tmp_path / "out"), NODE_RANK="0", NODE_SCRIPT=str(fake),
               RESTART_DELAY="0", MAX_RESTARTS="3")
    r = subprocess.run([str(ROOT / "launch/scaling/watchdog.sh"), "cfg.json"], env=env, capture_output=True,
                       text=True, timeout=60)
    return r.returncode, json.loads(plan.read_text())


def test_watchdog_restarts_until_terminal_phase(tmp_path):
    code, left = _watchdog(tmp_path, ["", "", "training_complete", "unused"])
    assert code == 0 and left == ["unused"]


def test_watchdog_never_retries_nonfinite(tmp_path):
    code, left = _watchdog(tmp_path, ["nonfinite", "unused"])
    assert code == 3 and left == ["unused"]


def test_watchdog_gives_up(tmp_path):
    code, left = _watchdog(tmp_path, ["", "", "", "", "", ""])
    assert code == 1 and len(left) == 2
