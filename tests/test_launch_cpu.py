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


def _fake_s3(tmp_path):
    """A stand-in for the storage CLI: s3://bucket/... maps to a local directory."""
    bucket = tmp_path / "bucket"
    bucket.mkdir()
    tool = tmp_path / "fake_s3"
    tool.write_text(f"""#!/usr/bin/env bash
set -e
loc() {{ echo "{bucket}/${{1#s3://}}"; }}
case "$1" in
  cp) dst="$(loc "$3")"; mkdir -p "$dst"; cp $2 "$dst" ;;
  ls) d="$(loc "$2")"; [ -d "$d" ] && for x in "$d"/*/; do [ -d "$x" ] && echo "DIR $(basename "$x")/"; done; true ;;
  rm) p="$(loc "$2")"; rm -f $p; rmdir "$(dirname "$p")" 2>/dev/null || true ;;
esac
""")
    tool.chmod(0o755)
    return bucket, tool


def test_s3_sync_mirrors_complete_checkpoints_and_prunes(tmp_path):
    bucket, tool = _fake_s3(tmp_path)
    out = tmp_path / "run"
    for step, complete in ((10, True), (20, True), (30, True), (40, True), (50, False)):
        d = out / f"checkpoint_{step:08d}" / "node_000"
        d.mkdir(parents=True)
        (d / "model.pt").write_text(str(step))
        if complete:
            (d / "complete.json").write_text("{}")
    (out / "metrics.jsonl").write_text("{}\n")
    env = dict(os.environ, OUTPUT_DIR=str(out), NODE_RANK="0", S3_PREFIX="s3://b/run", S3_TOOL=str(tool), ONCE="1",
               KEEP_REMOTE="2", MILESTONE_EVERY="20")
    subprocess.run([str(ROOT / "launch/scaling/s3_sync.sh")], env=env, check=True, timeout=60)
    remote = bucket / "b" / "run"
    kept = sorted(p.parent.parent.name for p in remote.glob("checkpoint_*/node_000/model.pt"))
    # 20 and 40 are milestones; of the rolling ones (10, 30) the newest KEEP_REMOTE=2 stay; 50 is incomplete
    assert kept == ["checkpoint_00000010", "checkpoint_00000020", "checkpoint_00000030", "checkpoint_00000040"]
    assert (remote / "records" / "metrics.jsonl").exists()
    assert (out / "checkpoint_00000010" / "node_000" / ".mirrored").exists()
    (out / "checkpoint_00000050" / "node_000" / "complete.json").write_text("{}")
    d = out / "checkpoint_00000070" / "node_000"
    d.mkdir(parents=True)
    (d / "model.pt").write_text("70")
    (d / "complete.json").write_text("{}")
    subprocess.run([str(ROOT / "launch/scaling/s3_sync.sh")], env=env, check=True, timeout=60)
    kept = sorted(p.parent.parent.name for p in remote.glob("checkpoint_*/node_000/model.pt"))
    assert kept == ["checkpoint_00000020", "checkpoint_00000040", "checkpoint_00000050", "checkpoint_00000070"]


def test_env_sh_exports_site_values(tmp_path):
    site = tmp_path / "site.json"
    site.write_text(json.dumps({"runtime_dir": str(tmp_path / "rt $(touch pwned)"), "micro_batch": 4}))
    script = f"source {ROOT / 'launch/env.sh'} --site-config {site}; echo \"$NEXTTRANSFORMER_RUNTIME|$NEXTTRANSFORMER_MICRO_BATCH\""
    out = subprocess.run(["bash", "-c", script], capture_output=True, text=True, check=True, cwd=tmp_path).stdout
    assert out.strip() == f"{tmp_path / 'rt $(touch pwned)'}|4"
    assert not (tmp_path / "pwned").exists()


def test_native_and_benchmark_launchers_dry_run():
    env = dict(os.environ, DRY_RUN="1", NNODES="2", NPROC_PER_NODE="8")
    out = subprocess.run([str(ROOT / "launch/native_train.sh"), "--config", "c.json"], env=env, capture_output=True,
                         text=True, check=True).stdout
    assert "nexttransformer_b200.native.train" in out and "--world-size 16" in out
    out = subprocess.run([str(ROOT / "launch/scaling/benchmark.sh"), "c.json"], env=dict(env, GPUS="4", STEPS="3"),
                         capture_output=True, text=True, check=True).stdout
    assert "--nproc-per-node 4" in out and "--benchmark 3" in out


def test_setup_environment_records_packages(tmp_path):
    """The set-up script resolves the site settings and records the package set; installing and
    building are skipped here (no index and no GPU needed)."""
    rt = tmp_path / "runtime"
    out = subprocess.run(["bash", str(ROOT / "launch/setup_environment.sh"), "--skip-install", "--no-build",
                          "--runtime-dir", str(rt)], capture_output=True, text=True, check=True).stdout
    assert "nexttransformer_b200 with torch" in out
    lock = (rt / "environment.lock.txt").read_text()
    assert "torch" in lock
    usage = subprocess.run(["bash", str(ROOT / "launch/setup_environment.sh"), "--help"], capture_output=True,
                           text=True, check=True).stdout
    assert "--wheelhouse" in usage
