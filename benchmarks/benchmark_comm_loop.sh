#!/usr/bin/env bash
# Pure ring-exchange sweep (the reference's ring/loop/benchmark_comm_loop.sh).
# Env: NP (2) SIZES ("262144 1048576 4194304 16777216") WARMUP (10) ITERS (100)
#      BACKENDS ("p2p ce nccl staged") TOKENS (set to sweep the bf16 K+V payload instead)
#      REFERENCE (0; 1 also runs the reference's own loop programs at the same sizes:
#      ring_loop_nccl and ring_loop_cuda_aware_Isendrecv, built unmodified by
#      benchmarks/build_reference.sh; their RESULT lines have the same format)
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
run_reference() {  # program, size
  timeout -k 30 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NP" \
    --master-addr 127.0.0.1 --master-port "$PORT" --no-python \
    "$PWD/baseline/_ref/bin/$1" "$2" "$WARMUP" "$ITERS" 2>&1 | grep RESULT | sed "s/^/reference /"
  PORT=$((PORT + 1))
}
if [[ -n "${TOKENS:-}" ]]; then
  for t in $TOKENS; do for b in $BACKENDS; do run 0 "$WARMUP" "$ITERS" --backend "$b" --payload-tokens "$t"; done; done
  SIZES=""
  for t in $TOKENS; do SIZES="$SIZES $((t * 8 * 128 * 2 * 2))"; done
else
  for s in $SIZES; do for b in $BACKENDS; do run "$s" "$WARMUP" "$ITERS" --backend "$b"; done; done
fi
if [[ "${REFERENCE:-0}" == 1 ]]; then
  [ -x baseline/_ref/bin/ring_loop_nccl ] || benchmarks/build_reference.sh
  for s in $SIZES; do
    for p in ring_loop_nccl ring_loop_cuda_aware_Isendrecv; do run_reference "$p" "$s"; done
  done
fi
