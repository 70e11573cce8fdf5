#!/usr/bin/env bash
#SBATCH --job-name=nexttransformer
#SBATCH --ntasks-per-node=1
#SBATCH --gpus-per-node=8
#SBATCH --exclusive
# One srun task per node; each starts that node's eight ranks through launch/train.sh.
#   sbatch --nodes=4 launch/slurm.sbatch --config configs/linear/gdn.json --output runs/gdn --formal --resume auto
set -euo pipefail
ROOT="${SLURM_SUBMIT_DIR:-$(pwd)}"
MASTER_ADDR="$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)"
export MASTER_ADDR MASTER_PORT="${MASTER_PORT:-29500}" NNODES="$SLURM_NNODES" NPROC_PER_NODE="${NPROC_PER_NODE:-8}"
srun --kill-on-bad-exit=1 bash -c 'NODE_RANK=$SLURM_NODEID exec "$0/launch/train.sh" "$@"' "$ROOT" "$@"
