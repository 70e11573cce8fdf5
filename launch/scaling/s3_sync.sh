#!/usr/bin/env bash
# Mirror this node's complete scaling checkpoints to object storage; node 0 also mirrors the run records.
# Remote retention follows the trainer's: every milestone checkpoint plus the newest KEEP_REMOTE rolling ones.
#   OUTPUT_DIR=runs/x NODE_RANK=0 S3_PREFIX=s3://bucket/prefix/run launch/scaling/s3_sync.sh
# Optional: SYNC_INTERVAL seconds between passes (600), KEEP_REMOTE (3), MILESTONE_EVERY updates (10000),
# ONCE=1 for a single pass, S3_TOOL (s5cmd; any tool with `cp SRC DST`, `ls PREFIX/` and `rm PATTERN`).
# A checkpoint is uploaded only once its node manifest (complete.json) exists, and marked .mirrored after
# a successful upload; a failed upload is retried on the next pass.
set -uo pipefail
: "${OUTPUT_DIR:?}" "${NODE_RANK:?}" "${S3_PREFIX:?}"
tool="${S3_TOOL:-s5cmd}"
node="node_$(printf %03d "$NODE_RANK")"
keep="${KEEP_REMOTE:-3}"; every="${MILESTONE_EVERY:-10000}"

upload_complete() {
  local manifest dir name
  for manifest in "$OUTPUT_DIR"/checkpoint_*/"$node"/complete.json; do
    [[ -e "$manifest" ]] || continue
    dir="$(dirname "$manifest")"; name="$(basename "$(dirname "$dir")")"
    [[ -e "$dir/.mirrored" ]] && continue
    if "$tool" cp "$dir/*" "$S3_PREFIX/$name/$node/"; then touch "$dir/.mirrored"
    else echo "s3_sync: upload of $name failed; retrying next pass" >&2; fi
  done
}

upload_records() {
  local f
  for f in "$OUTPUT_DIR"/*.json "$OUTPUT_DIR"/*.jsonl; do
    [[ -e "$f" ]] && { "$tool" cp "$f" "$S3_PREFIX/records/" || echo "s3_sync: record $f not uploaded" >&2; }
  done
}

prune_remote() {
  # remote checkpoint names, oldest first; milestones are never removed
  local names=() rolling=() name step i
  mapfile -t names < <("$tool" ls "$S3_PREFIX/" 2>/dev/null | awk '$1 == "DIR" {print $2}' |
                       sed -n 's|^\(checkpoint_[0-9]*\)/$|\1|p' | sort)
  for name in "${names[@]}"; do
    step=$((10#${name#checkpoint_}))
    (( step % every )) && rolling+=("$name")
  done
  for (( i = 0; i < ${#rolling[@]} - keep; i++ )); do
    "$tool" rm "$S3_PREFIX/${rolling[i]}/$node/*" || echo "s3_sync: could not remove ${rolling[i]}" >&2
  done
}

while true; do
  upload_complete
  [[ "$NODE_RANK" == 0 ]] && upload_records
  prune_remote
  [[ "${ONCE:-0}" == 1 ]] && break
  sleep "${SYNC_INTERVAL:-600}"
done
