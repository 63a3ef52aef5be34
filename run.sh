#!/usr/bin/env bash
# Build libgemm.so (sm_100a) and run the bench, like the reference's run.sh:
#   ./run.sh [flags]            (flags as mlp_bench.py; default: the suite)
set -euo pipefail
ROOT="$(cd "$(dirname "$0")" && pwd)"
cd "$ROOT"
echo "== hardware =="
nvidia-smi --query-gpu=name,memory.total,clocks.max.sm --format=csv,noheader 2>/dev/null || true
echo "== compile libgemm.so (sm_100a) =="
make -s -C fp8-mlp-metal41-bench_b200
echo "== run =="
exec python mlp_bench.py "$@"
