#!/usr/bin/env bash
# Scheduler-model presets (the reference's workload/run_experiments.sh):
# tables 4/5/6 with the alpha/beta pairs calibrated from single-GPU timings.
set -euo pipefail
cd "$(dirname "$0")/.."
make -s build/bin/rattn_demo
DEMO=./build/bin/rattn_demo
header() {
  printf "%-6s %-5s %-6s %-6s | %-10s %-6s | %-10s %-6s | %-10s %-6s | %-10s %-6s | %-10s\n" \
    "seq" "GPUs" "mask" "blocks" "RR(ms)" "imb" "BlkLPT" "imb" "RowLPT" "imb" "DP(ms)" "imb" "ideal"
  echo "-----------------------------------------------------------------------------------------------------------"
}
echo "====== Table 4: Varying seq, 2 GPUs, causal ======"
header
$DEMO --seq  512 --gpus 2 --mask causal --alpha 0.169 --beta 0.00000694
$DEMO --seq 1024 --gpus 2 --mask causal --alpha 1.21  --beta 0.00000384
$DEMO --seq 2048 --gpus 2 --mask causal --alpha 1.21  --beta 0.00000384
$DEMO --seq 4096 --gpus 2 --mask causal --alpha 1.21  --beta 0.00000384
echo ""
echo "====== Table 5: Varying GPUs, seq=4096, causal ======"
header
for g in 2 3 4 8; do $DEMO --seq 4096 --gpus $g --mask causal --alpha 1.21 --beta 0.00000384; done
echo ""
echo "====== Table 6: Causal vs Full, seq=4096, 2 GPUs ======"
header
$DEMO --seq 4096 --gpus 2 --mask full   --alpha 1.21  --beta 0.00000384
$DEMO --seq 4096 --gpus 2 --mask causal --alpha 1.21  --beta 0.00000384
