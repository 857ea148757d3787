#!/usr/bin/env bash
# Ring-attention backend sweep (the reference's ring/attention/bench/benchmark_attention.sh).
# Env: NP (2) SIZES ("262144 524288 1048576") WARMUP (10) ITERS (100) NUMERICS (fp32|bf16)
set -euo pipefail
cd "$(dirname "$0")/.."
export PYTHONPATH="$PWD${PYTHONPATH:+:$PYTHONPATH}"
NP=${NP:-2}
SIZES=${SIZES:-"262144 524288 1048576"}
WARMUP=${WARMUP:-10}
ITERS=${ITERS:-100}
NUMERICS=${NUMERICS:-fp32}
PORT=${PORT:-29541}
if [[ "$NUMERICS" == bf16 ]]; then BACKENDS=${BACKENDS:-"fused nccl"}; EXTRA=(--numerics bf16 --init randn --heads 8);
else BACKENDS=${BACKENDS:-"nccl staged"}; EXTRA=(); fi
for size in $SIZES; do
  for b in $BACKENDS; do
    echo "== size=$size backend=$b"
    timeout -k 30 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NP" \
      --master-addr 127.0.0.1 --master-port "$PORT" \
      -m multi_gpu_flashattention_b200.benchmarks.ring_attention "$size" "$WARMUP" "$ITERS" \
      --backend "$b" "${EXTRA[@]}" 2>&1 | grep -E "bench:|avg_total"
    PORT=$((PORT + 1))
  done
done
