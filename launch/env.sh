#!/usr/bin/env bash
# Source this file to export the resolved machine settings into the current shell:
#   source launch/env.sh [--site-config site.json] [--runtime-dir D] [--data-dir D] ...
# The site JSON is parsed as data by runtime/site.py and every value is shell-quoted; nothing in it runs.
_nt_root="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
_nt_exports="$(cd "$_nt_root" && "${PYTHON:-python3}" -m nexttransformer_b200.runtime.site --shell "$@")" || return $?
eval "$_nt_exports"
unset _nt_exports _nt_root
