#!/usr/bin/env bash
# Start this node's ranks of a scaling run (NNODES=1 for one node).
#   NNODES=N NODE_RANK=K MASTER_ADDR=HOST MASTER_PORT=PORT launch/scaling/node.sh CONFIG [training options]
# Optional: GPUS (8), MICRO_BATCH (2), OUTPUT_DIR, PYTHON (python), SCALING_ENV (a file of site exports kept
# outside the repository: network settings, tracking key).
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)"
if [[ $# == 0 || " $* " == *" --help "* ]]; then
  echo 'usage: NNODES=N NODE_RANK=K MASTER_ADDR=HOST MASTER_PORT=PORT launch/scaling/node.sh CONFIG [options]'
  exit 0
fi
CONFIG="$1"; shift
if [[ -n "${SCALING_ENV:-}" ]]; then source "$SCALING_ENV"; fi
: "${NNODES:?}" "${NODE_RANK:?}" "${MASTER_ADDR:?}" "${MASTER_PORT:?}"
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
OUTPUT="${OUTPUT_DIR:-runs/scaling_$(basename "$CONFIG" .json)}"
cd "$ROOT"
exec "${PYTHON:-python}" -m torch.distributed.run --nnodes="$NNODES" --node-rank="$NODE_RANK" \
  --nproc-per-node="${GPUS:-8}" --master-addr="$MASTER_ADDR" --master-port="$MASTER_PORT" \
  -m nexttransformer_b200.scaling.train --config "$CONFIG" --output "$OUTPUT" --micro-batch "${MICRO_BATCH:-2}" "$@"
