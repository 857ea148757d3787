#!/usr/bin/env bash
# One-shot legacy ring correctness (the reference's
# ring/attention/gpu/check_attention_gpu_correctness.sh, on torchrun + this
# framework): run the one-shot ring with each transport (and the host-attention
# ring), check every dump against the full single-device reference with
# verify_full, and compare the runs pairwise (PASS iff max_abs <= ABS_TOL or
# max_rel <= REL_TOL).
#
# Env: NP (2) SEQ (1024 tokens per rank) ABS_TOL (1e-3) REL_TOL (1e-5)
#      RESULTS_ROOT (results) RUN_LABEL (timestamp) CHECK_P2P (1) CHECK_CPU (1)
#      NATIVE (0; 1 runs build/bin/ring_oneshot instead of the Python driver)
#      REFERENCE (0; 1 also runs the reference's own one-shot programs,
#      gpu/ring_attention_{staged,cuda_aware,nccl}_gpu built unmodified by
#      benchmarks/build_reference.sh, seq 1024 only, and compares their dumps)
set -euo pipefail
cd "$(dirname "$0")/.."
export PYTHONPATH="$PWD${PYTHONPATH:+:$PYTHONPATH}"
NP=${NP:-2}
SEQ=${SEQ:-1024}
SIZE=$((SEQ * 64 * 4))
ABS_TOL=${ABS_TOL:-1e-3}
REL_TOL=${REL_TOL:-1e-5}
CHECK_P2P=${CHECK_P2P:-1}
CHECK_CPU=${CHECK_CPU:-1}
RESULTS_ROOT=${RESULTS_ROOT:-results}
RUN_LABEL=${RUN_LABEL:-gpu_correctness_$(date +%Y%m%d_%H%M%S)}
OUT="$RESULTS_ROOT/$RUN_LABEL/gpu_attention_correctness_np$NP"
PORT=${PORT:-29571}
mkdir -p "$OUT"
make -s build/bin/verify_full

echo "========== GPU Attention Correctness Check (one-shot) =========="
echo "np=$NP seq=$SEQ kv_size=$SIZE results=$OUT"

run_backend() {  # label, args...
  local label=$1; shift
  local dir="$OUT/$label"
  mkdir -p "$dir"
  echo ""
  echo "===== gpu backend=$label ====="
  if [[ "${NATIVE:-0}" == 1 ]]; then
    local prog=(--no-python "$PWD/build/bin/ring_oneshot")
  else
    local prog=(-m multi_gpu_flashattention_b200.benchmarks.ring_oneshot)
  fi
  timeout -k 30 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NP" \
      --master-addr 127.0.0.1 --master-port "$PORT" \
      "${prog[@]}" --seq "$SEQ" --out-dir "$dir" "$@" \
      2>&1 | tee "$dir/run.log" | grep -E "step|done" || true
  PORT=$((PORT + 1))
  echo "--- full reference check: $label ---"
  ./build/bin/verify_full "$dir" "$NP" "$SIZE" | tee "$dir/verify.log" | tail -1
}

compare_pair() {  # name, dirA, dirB
  python - "$1" "$2" "$3" "$NP" "$ABS_TOL" "$REL_TOL" <<'PY'
import sys
import numpy as np
name, a, b, npr, atol, rtol = sys.argv[1], sys.argv[2], sys.argv[3], int(sys.argv[4]), float(sys.argv[5]), float(sys.argv[6])
tot = 0; sabs = 0.0; mabs = 0.0; mrel = 0.0; worst = -1
for r in range(npr):
    x = np.fromfile(f"{a}/ring_output_rank{r}.bin", dtype="<f4").astype(np.float64)
    y = np.fromfile(f"{b}/ring_output_rank{r}.bin", dtype="<f4").astype(np.float64)
    if x.shape != y.shape:
        raise SystemExit(f"rank {r}: length mismatch {x.size} vs {y.size}")
    d = np.abs(x - y)
    rel = d / np.maximum(np.maximum(np.abs(x), np.abs(y)), 1e-12)
    tot += d.size; sabs += d.sum()
    if d.max() > mabs: mabs, worst = d.max(), r
    mrel = max(mrel, rel.max())
ok = mabs <= atol or mrel <= rtol
print(f"{name}: {'PASS' if ok else 'FAIL'} elements={tot} max_abs_err={mabs:.6e} "
      f"mean_abs_err={sabs / max(tot, 1):.6e} max_rel_err={mrel:.6e} worst_rank={worst} "
      f"abs_tol={atol:.1e} rel_tol={rtol:.1e}")
sys.exit(0 if ok else 1)
PY
}

run_backend staged --backend staged
run_backend nccl --backend nccl
compare_pair staged_vs_nccl "$OUT/staged" "$OUT/nccl"
if [[ "$CHECK_P2P" == 1 ]]; then
  run_backend p2p --backend p2p
  compare_pair staged_vs_p2p "$OUT/staged" "$OUT/p2p"
fi
if [[ "$CHECK_CPU" == 1 ]]; then
  run_backend cpu_staged --attention cpu --backend staged
  compare_pair gpu_vs_cpu_attention "$OUT/staged" "$OUT/cpu_staged"
fi
if [[ "${REFERENCE:-0}" == 1 && "$SEQ" == 1024 ]]; then
  [ -x baseline/_ref/bin/ring_attention_nccl_gpu ] || benchmarks/build_reference.sh
  for prog in staged cuda_aware nccl; do
    dir="$OUT/reference_$prog"
    mkdir -p "$dir"
    echo ""
    echo "===== reference program ring_attention_${prog}_gpu ====="
    (cd "$dir" && timeout -k 30 600 python -m torch.distributed.run --nnodes=1 \
        --nproc-per-node "$NP" --master-addr 127.0.0.1 --master-port "$PORT" --no-python \
        "$OLDPWD/baseline/_ref/bin/ring_attention_${prog}_gpu" 2>&1 | tee run.log \
        | grep -E "step|done" || true)
    PORT=$((PORT + 1))
    ./build/bin/verify_full "$dir" "$NP" "$SIZE" | tee "$dir/verify.log" | tail -1
    compare_pair "staged_vs_reference_$prog" "$OUT/staged" "$dir"
  done
fi
echo ""
echo "========== GPU Correctness Check Done =========="
