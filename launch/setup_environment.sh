#!/usr/bin/env bash
# Prepare a machine to run the framework: resolve the site settings (launch/env.sh), optionally create
# a virtual environment and install the Python packages of launch/requirements.txt (from an index or an
# offline wheelhouse), build the sm_100a extensions in place, check that the package and its kernels
# load, and record the resulting package set under the runtime directory.
#
#   launch/setup_environment.sh [--site-config F] [--runtime-dir D] [other site options]
#                               [--venv DIR] [--wheelhouse DIR] [--index-url URL]
#                               [--skip-install] [--no-build]
set -euo pipefail
REPO_ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
VENV="" WHEELHOUSE="" INDEX_URL="" SKIP_INSTALL=0 BUILD=1
SITE_ARGS=()
while [[ $# -gt 0 ]]; do
  case "$1" in
    --help) sed -n '2,9p' "${BASH_SOURCE[0]}"; exit 0 ;;
    --venv) VENV="$2"; shift 2 ;;
    --wheelhouse) WHEELHOUSE="$2"; shift 2 ;;
    --index-url) INDEX_URL="$2"; shift 2 ;;
    --skip-install) SKIP_INSTALL=1; shift ;;
    --no-build) BUILD=0; shift ;;
    *) SITE_ARGS+=("$1"); shift ;;
  esac
done
source "$REPO_ROOT/launch/env.sh" "${SITE_ARGS[@]}"
PY="${PYTHON:-python3}"
if [[ -n "$VENV" ]]; then
  # the venv sees the system's packages, so an image that already carries torch keeps it
  [[ -x "$VENV/bin/python" ]] || "$PY" -m venv --system-site-packages "$VENV"
  PY="$VENV/bin/python"
fi
if [[ "$SKIP_INSTALL" == 0 ]]; then
  PIP_ARGS=(install -r "$REPO_ROOT/launch/requirements.txt")
  if [[ -n "$WHEELHOUSE" ]]; then PIP_ARGS+=(--no-index --find-links "$WHEELHOUSE"); fi
  if [[ -n "$INDEX_URL" ]]; then PIP_ARGS+=(--index-url "$INDEX_URL"); fi
  "$PY" -m pip "${PIP_ARGS[@]}"
fi
cd "$REPO_ROOT"
if [[ "$BUILD" == 1 ]]; then
  "$PY" -m nexttransformer_b200.build
  "$PY" -c "from nexttransformer_b200.ops._ext import ext; ext(); print('sm_100a extensions load')"
fi
"$PY" -c "import nexttransformer_b200, torch; print('nexttransformer_b200 with torch', torch.__version__)"
mkdir -p "$NEXTTRANSFORMER_RUNTIME"
"$PY" -m pip freeze > "$NEXTTRANSFORMER_RUNTIME/environment.lock.txt"
echo "environment recorded in $NEXTTRANSFORMER_RUNTIME/environment.lock.txt"
