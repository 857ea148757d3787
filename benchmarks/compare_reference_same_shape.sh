#!/usr/bin/env bash
# Same-shape comparison with the reference's own program: its NCCL ring
# attention (fp32, one head, head_dim 64, non-causal, K=V; built unmodified by
# benchmarks/build_reference.sh) against this framework's ring at the same
# tokens per rank and world size: the fp32 reference-numerics kernels over NCCL
# (same maths, same inputs) and the bf16 fused ring (one head, head_dim 64,
# non-causal). Prints the reference's avg line and one JSON line per backend of
# ours, for every size in SIZES (bytes of one rank's fp32 KV shard, multiples
# of 256).
# Env: NP (2) SIZES ("262144 1048576 4194304") WARMUP (3) ITERS (10)
set -euo pipefail
cd "$(dirname "$0")/.."
NP=${NP:-2}
SIZES=${SIZES:-"262144 1048576 4194304"}
WARMUP=${WARMUP:-3}
ITERS=${ITERS:-10}
PORT=${PORT:-29671}
REF="$PWD/baseline/_ref/bin/ring_attention_nccl_gpu_bench"
[ -x "$REF" ] || benchmarks/build_reference.sh
make -s cuda-tools
run() {  # label, program, args...
  local label=$1; shift
  echo "== np=$NP $label"
  timeout -k 30 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NP" \
    --master-addr 127.0.0.1 --master-port "$PORT" --no-python "$@" 2>&1 \
    | grep -E '^\{|avg_total' || true
  PORT=$((PORT + 1))
}
for s in $SIZES; do
  run "size=$s reference nccl (fp32)" "$REF" "$s" "$WARMUP" "$ITERS"
  run "size=$s ours nccl (fp32 reference numerics)" build/bin/ring_attention_bench "$s" \
    "$WARMUP" "$ITERS" --backend nccl --json
  run "size=$s ours fused (bf16, 1 head x d64)" build/bin/ring_attention_bench "$s" \
    "$WARMUP" "$ITERS" --numerics bf16 --init randn --heads 1 --head-dim 64 \
    --layout contiguous --backend fused --json
done
