#!/usr/bin/env bash
# torchrun launcher of the native-track trainer (SSSL Dense, MoR, LoopFormer, Circle) on one node, or on each
# node of a multi-node job:
#   launch/native_train.sh --config configs/native/mor.json --data bestfit --core BUNDLE
# Environment: NNODES (1), NPROC_PER_NODE (8), NODE_RANK (0), MASTER_ADDR (127.0.0.1), MASTER_PORT (29500),
# PYTHON (python), DRY_RUN=1 prints the command instead of running it.
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
NNODES="${NNODES:-1}"; NPROC="${NPROC_PER_NODE:-8}"; NODE_RANK="${NODE_RANK:-0}"
CMD=("${PYTHON:-python}" -m torch.distributed.run --nnodes "$NNODES" --node-rank "$NODE_RANK" --nproc-per-node "$NPROC"
     --master-addr "${MASTER_ADDR:-127.0.0.1}" --master-port "${MASTER_PORT:-29500}"
     -m nexttransformer_b200.native.train --world-size "$((NNODES * NPROC))" "$@")
if [[ "${DRY_RUN:-0}" == 1 ]]; then printf '%q ' "${CMD[@]}"; echo; exit 0; fi
cd "$ROOT"
export PYTORCH_CUDA_ALLOC_CONF="${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}"
exec "${CMD[@]}"
