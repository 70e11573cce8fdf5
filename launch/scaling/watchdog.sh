#!/usr/bin/env bash
# Keep this node's share of a scaling run going: every launch resumes from the newest checkpoint complete on
# every node; the loop ends when the trainer writes a terminal phase into this node's status file written
# after the launch started.  A non-finite loss or gradient is never retried (exit 3).
#   OUTPUT_DIR=DIR NNODES=N NODE_RANK=K MASTER_ADDR=HOST MASTER_PORT=PORT launch/scaling/watchdog.sh CONFIG [options]
# Optional: MAX_RESTARTS (20), RESTART_DELAY seconds (60), NODE_SCRIPT (launch/scaling/node.sh).
set -uo pipefail
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)"
if [[ $# == 0 || " $* " == *" --help "* ]]; then
  echo 'usage: OUTPUT_DIR=DIR NNODES=N NODE_RANK=K MASTER_ADDR=HOST MASTER_PORT=PORT launch/scaling/watchdog.sh CONFIG [options]'
  exit 0
fi
CONFIG="$1"; shift
: "${OUTPUT_DIR:?set OUTPUT_DIR so every launch uses the same run directory}" "${NODE_RANK:?}"
STATUS="$OUTPUT_DIR/status.node$(printf %03d "$NODE_RANK").json"
NODE_SCRIPT="${NODE_SCRIPT:-$ROOT/launch/scaling/node.sh}"
restarts=0
while true; do
  started="$(date +%s)"
  "$NODE_SCRIPT" "$CONFIG" --resume auto "$@"
  code=$?
  phase="$(python3 - "$STATUS" "$started" <<'PY'
import json, os, sys
path, since = sys.argv[1], float(sys.argv[2])
fresh = os.path.exists(path) and os.path.getmtime(path) >= since
print(json.load(open(path))["phase"] if fresh else "")
PY
)"
  case "$phase" in
    training_complete|smoke_complete|stopped) echo "watchdog: $phase"; exit 0 ;;
    nonfinite) echo "watchdog: non-finite loss or gradient; not restarting" >&2; exit 3 ;;
  esac
  restarts=$((restarts + 1))
  if (( restarts > ${MAX_RESTARTS:-20} )); then echo "watchdog: giving up after $restarts failed launches" >&2; exit 1; fi
  echo "watchdog: launch exited with $code; restart $restarts of ${MAX_RESTARTS:-20} in ${RESTART_DELAY:-60}s" >&2
  sleep "${RESTART_DELAY:-60}"
done
