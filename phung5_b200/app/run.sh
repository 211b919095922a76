#!/usr/bin/env bash
# Boot the generation service: host limits, preflight, local engines, HTTP API (see boot.py).
#   PHX_APP_CONFIG=configs/pipeline.yaml phung5_b200/app/run.sh [--skip-preflight] [--no-spawn]
set -euo pipefail
ulimit -n "$(ulimit -Hn)" 2>/dev/null || true
export OMP_NUM_THREADS="${OMP_NUM_THREADS:-1}"
cd "$(dirname "$0")/../.."
exec python -m phung5_b200.app.boot --config "${PHX_APP_CONFIG:-configs/pipeline.yaml}" "$@"
