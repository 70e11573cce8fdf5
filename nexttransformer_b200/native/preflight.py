"""Bounded multi-GPU preflight of a native configuration: run the benchmark with the full routed
path at a micro-batch, halve it on out-of-memory (the global batch stays fixed), and record the
first size that fits.  Refuses to start while other compute processes hold the GPUs.  Each attempt
runs in its own process group under a timeout and is killed as a group if it overruns.
Behaviour: ``nexttransformer/native/preflight.py:14-61``.
"""
from nexttransformer_b200.runtime.site import add_runtime_arguments, bootstrap_runtime

if __name__ == "__main__":
    bootstrap_runtime()

import argparse
import json
import os
from pathlib import Path
import signal
import subprocess
import sys


def attempt_command(config, batch, result, gpus):
    return [sys.executable, "-m", "torch.distributed.run", "--standalone", f"--nproc_per_node={gpus}",
            "-m", "nexttransformer_b200.native.benchmark", "--config", str(config), "--micro-batch", str(batch),
            "--warmup", "2", "--steps", "2", "--stress-full-path", "--output", str(result)]


def run_attempt(command, log, timeout):
    with open(log, "w") as out:
        worker = subprocess.Popen(command, stdout=out, stderr=subprocess.STDOUT, start_new_session=True,
                                  env={**os.environ, "WANDB_MODE": "disabled"})
        try:
            return worker.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            os.killpg(worker.pid, signal.SIGTERM)
            try:
                worker.wait(timeout=20)
            except subprocess.TimeoutExpired:
                os.killpg(worker.pid, signal.SIGKILL)
                worker.wait()
            raise RuntimeError(f"preflight timed out; inspect {log}")


def main(argv=None, runner=run_attempt, busy=None):
    p = argparse.ArgumentParser(description=__doc__, allow_abbrev=False)
    add_runtime_arguments(p)
    p.add_argument("--config", type=Path, required=True)
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--gpus", type=int, default=8)
    p.add_argument("--timeout", type=int, default=1800)
    a = p.parse_args(argv)
    from nexttransformer_b200.runtime.site import resolve
    resolve(a)
    from nexttransformer_b200.models.native.config import load_config
    from nexttransformer_b200.runtime.files import atomic_json
    mc, tc = load_config(a.config)
    if busy is None:
        busy = subprocess.check_output(["nvidia-smi", "--query-compute-apps=pid", "--format=csv,noheader,nounits"],
                                       text=True).strip()
    if busy:
        raise RuntimeError("GPU compute processes already exist; preflight will not interrupt them")
    a.output.parent.mkdir(parents=True, exist_ok=True)
    if a.output.exists():
        raise ValueError("preflight output already exists")
    batch = a.micro_batch or 8
    attempts = []
    while batch >= 1:
        tc.accumulation(mc, a.gpus, batch)
        result = a.output.with_name(a.output.stem + f"_b{batch}.json")
        log = result.with_suffix(".log")
        code = runner(attempt_command(a.config, batch, result, a.gpus), log, a.timeout)
        attempts.append({"micro_batch": batch, "exit_code": code, "log": str(log)})
        if code == 0:
            atomic_json(a.output, {"status": "passed", "micro_batch": batch,
                                   "accumulation": tc.accumulation(mc, a.gpus, batch),
                                   "global_batch_tokens": tc.global_batch_tokens, "attempts": attempts,
                                   "evidence": json.loads(result.read_text())})
            print(f"PREFLIGHT PASSED: --micro-batch {batch}; accumulation {tc.accumulation(mc, a.gpus, batch)}")
            return batch
        text = Path(log).read_text()
        if "out of memory" not in text.lower() and "OutOfMemoryError" not in text:
            raise RuntimeError(f"preflight failed for a reason other than OOM; inspect {log}")
        batch //= 2
    atomic_json(a.output, {"status": "failed", "attempts": attempts})
    raise RuntimeError("even micro-batch 1 did not fit")


if __name__ == "__main__":
    main()
