#!/usr/bin/env bash
# Fusion ablation at one world size: the same bf16 causal ring (zigzag shards,
# HEADS x 128, SEQ tokens in total) with the transport fused into the attention
# kernel, as a separate push kernel, on the copy engine, and over NCCL
# (native ring_attention_bench; one JSON line per backend, appended to OUT).
# Env: NP (2) SEQ (131072) HEADS (32) WARMUP (2) ITERS (5)
#      BACKENDS ("fused p2p_unfused ce_unfused nccl") TAG_CHECK (1) OUT (results/ablation.jsonl)
set -euo pipefail
cd "$(dirname "$0")/.."
NP=${NP:-2}
SEQ=${SEQ:-131072}
HEADS=${HEADS:-32}
WARMUP=${WARMUP:-2}
ITERS=${ITERS:-5}
BACKENDS=${BACKENDS:-"fused p2p_unfused ce_unfused nccl"}
OUT=${OUT:-results/ablation.jsonl}
PORT=${PORT:-29651}
make -s cuda-tools
mkdir -p "$(dirname "$OUT")"
SIZE=$((SEQ / NP * HEADS * 128 * 4))   # kv_size: tokens per rank x heads x 128 x 4 bytes
for b in $BACKENDS; do
  echo "== np=$NP seq=$SEQ backend=$b"
  MGFA_TAG_CHECK=${TAG_CHECK:-1} timeout -k 30 600 python -m torch.distributed.run --nnodes=1 \
    --nproc-per-node "$NP" --master-addr 127.0.0.1 --master-port "$PORT" --no-python \
    build/bin/ring_attention_bench "$SIZE" "$WARMUP" "$ITERS" --numerics bf16 --init randn \
    --causal --layout zigzag --heads "$HEADS" --backend "$b" --json 2>&1 \
    | grep -E '^\{' | tee -a "$OUT"
  PORT=$((PORT + 1))
done
