#!/usr/bin/env bash
# Pure ring-exchange sweep (the reference's ring/loop/benchmark_comm_loop.sh).
# Env: NP (2) SIZES ("262144 1048576 4194304 16777216") WARMUP (10) ITERS (100)
#      BACKENDS ("p2p ce nccl staged") TOKENS (set to sweep the bf16 K+V payload instead)
set -euo pipefail
cd "$(dirname "$0")/.."
export PYTHONPATH="$PWD${PYTHONPATH:+:$PYTHONPATH}"
NP=${NP:-2}
SIZES=${SIZES:-"262144 1048576 4194304 16777216"}
WARMUP=${WARMUP:-10}
ITERS=${ITERS:-100}
BACKENDS=${BACKENDS:-"p2p ce nccl staged"}
PORT=${PORT:-29551}
run() {
  timeout -k 30 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NP" \
    --master-addr 127.0.0.1 --master-port "$PORT" \
    -m multi_gpu_flashattention_b200.benchmarks.ring_loop "$@" 2>&1 | grep RESULT
  PORT=$((PORT + 1))
}
if [[ -n "${TOKENS:-}" ]]; then
  for t in $TOKENS; do for b in $BACKENDS; do run 0 "$WARMUP" "$ITERS" --backend "$b" --payload-tokens "$t"; done; done
else
  for s in $SIZES; do for b in $BACKENDS; do run "$s" "$WARMUP" "$ITERS" --backend "$b"; done; done
fi
