#!/usr/bin/env bash
# torchrun launcher of the formal / research trainer on one node, or on each node of a multi-node job.
#   launch/train.sh --config configs/baseline/dense_full.json --output runs/dense_full --formal
# Environment: NNODES (1), NPROC_PER_NODE (8), NODE_RANK (0), MASTER_ADDR (127.0.0.1), MASTER_PORT (29500),
# PYTHON (python), DRY_RUN=1 prints the command.  Formal and research runs use 8, 16 or 32 ranks in total;
# a --smoke-steps run may use any number.
set -euo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
NNODES="${NNODES:-1}"; NPROC="${NPROC_PER_NODE:-8}"; NODE_RANK="${NODE_RANK:-0}"
ADDR="${MASTER_ADDR:-127.0.0.1}"; PORT="${MASTER_PORT:-29500}"; PYTHON="${PYTHON:-python}"
WORLD=$((NNODES * NPROC))
case " $* " in *" --smoke-steps"*) smoke=1 ;; *) smoke=0 ;; esac
if [[ $smoke == 0 && $WORLD != 8 && $WORLD != 16 && $WORLD != 32 ]]; then
  echo "train.sh: $NNODES node(s) x $NPROC GPU(s) = $WORLD ranks; formal and research runs use 8, 16 or 32" >&2
  exit 2
fi
CMD=("$PYTHON" -m torch.distributed.run --nnodes "$NNODES" --node-rank "$NODE_RANK" --nproc-per-node "$NPROC"
     --master-addr "$ADDR" --master-port "$PORT" -m nexttransformer_b200.train "$@")
if [[ "${DRY_RUN:-0}" == 1 ]]; then printf '%q ' "${CMD[@]}"; echo; exit 0; fi
cd "$ROOT"
exec "${CMD[@]}"
