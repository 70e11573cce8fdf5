#!/usr/bin/env bash
# Throughput of one scaling configuration on this node: a few timed updates through the scaling trainer's
# benchmark path, one JSON line per run.
#   GPUS=8 STEPS=10 launch/scaling/benchmark.sh configs/scaling/t3_dense_l20.json [--micro-batch 2]
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)"
if [[ $# == 0 ]]; then echo 'usage: GPUS=N launch/scaling/benchmark.sh CONFIG [options]'; exit 2; fi
CONFIG="$1"; shift
CMD=("${PYTHON:-python}" -m torch.distributed.run --standalone --local-addr 127.0.0.1 --nproc-per-node "${GPUS:-8}"
     -m nexttransformer_b200.scaling.train --config "$CONFIG" --benchmark "${STEPS:-10}" "$@")
if [[ "${DRY_RUN:-0}" == 1 ]]; then printf '%q ' "${CMD[@]}"; echo; exit 0; fi
cd "$ROOT"
exec "${CMD[@]}"
