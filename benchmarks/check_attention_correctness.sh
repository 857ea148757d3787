#!/usr/bin/env bash
# Ring-attention correctness pipeline (the reference's
# ring/attention/bench/check_attention_correctness.sh, on torchrun + this
# framework): run backend pairs with ATTENTION_DUMP_OUTPUT=1, check every dump
# against the full single-device reference with verify_full, and compare each
# pair element-wise (PASS iff max_abs <= ABS_TOL or max_rel <= REL_TOL).
#
# Env: NP (2) SIZE (262144) WARMUP (1) ITERS (1) ABS_TOL (1e-3) REL_TOL (1e-5)
#      RESULTS_ROOT (results) RUN_LABEL (timestamp) INIT (legacy|randn) CHECK_P2P (1)
#      CHECK_REFERENCE (1 when baseline/_ref/bin holds the reference's programs,
#      built by benchmarks/build_reference.sh; legacy inputs only): also run the
#      reference's own NCCL and CUDA-aware overlap programs with dumps, check
#      them with verify_full, and compare this framework's dumps with theirs.
set -euo pipefail
cd "$(dirname "$0")/.."
export PYTHONPATH="$PWD${PYTHONPATH:+:$PYTHONPATH}"
NP=${NP:-2}
SIZE=${SIZE:-262144}
WARMUP=${WARMUP:-1}
ITERS=${ITERS:-1}
ABS_TOL=${ABS_TOL:-1e-3}
REL_TOL=${REL_TOL:-1e-5}
INIT=${INIT:-legacy}
RESULTS_ROOT=${RESULTS_ROOT:-results}
RUN_LABEL=${RUN_LABEL:-$(date +%Y%m%d_%H%M%S)}
OUT="$RESULTS_ROOT/$RUN_LABEL"
PORT=${PORT:-29531}
mkdir -p "$OUT"
make -s build/bin/verify_full
VERIFY_ARGS=()
[[ "$INIT" == randn ]] && VERIFY_ARGS=(--init randn)

run_bench() {  # label, extra args...
  local label=$1; shift
  local dir="$OUT/$label"
  mkdir -p "$dir"
  (cd "$dir" && ATTENTION_DUMP_OUTPUT=1 timeout -k 30 600 python -m torch.distributed.run \
      --nnodes=1 --nproc-per-node "$NP" --master-addr 127.0.0.1 --master-port "$PORT" \
      -m multi_gpu_flashattention_b200.benchmarks.ring_attention "$SIZE" "$WARMUP" "$ITERS" \
      --init "$INIT" "$@" > bench.log 2>&1)
  PORT=$((PORT + 1))
  ./build/bin/verify_full "$dir" "$NP" "$SIZE" "${VERIFY_ARGS[@]}" | tee "$dir/verify.log" | tail -1
}

compare_pair() {  # name, dirA, dirB
  python - "$1" "$2" "$3" "$NP" "$ABS_TOL" "$REL_TOL" <<'PY'
import sys
import numpy as np
name, a, b, npr, atol, rtol = sys.argv[1], sys.argv[2], sys.argv[3], int(sys.argv[4]), float(sys.argv[5]), float(sys.argv[6])
ok = True
for r in range(npr):
    x = np.fromfile(f"{a}/ring_output_rank{r}.bin", dtype="<f4")
    y = np.fromfile(f"{b}/ring_output_rank{r}.bin", dtype="<f4")
    if x.shape != y.shape or not (np.isfinite(x).all() and np.isfinite(y).all()):
        ok = False
        continue
    d = np.abs(x.astype(np.float64) - y)
    rel = d / np.maximum(np.maximum(np.abs(x), np.abs(y)), 1e-12)
    ok = ok and (d.max() <= atol or rel.max() <= rtol)
print(f"{name}: {'PASS' if ok else 'FAIL'}")
sys.exit(0 if ok else 1)
PY
}

run_bench nccl --backend nccl
run_bench nccl_overlap --backend nccl --overlap
run_bench staged --backend staged
run_bench staged_overlap --backend staged --overlap
compare_pair nccl_vs_overlap "$OUT/nccl" "$OUT/nccl_overlap"
compare_pair staged_vs_overlap "$OUT/staged" "$OUT/staged_overlap"
if [[ "${CHECK_P2P:-1}" == 1 ]]; then
  # the KV shard over NVLink: push kernel and copy engine (sequential order)
  run_bench p2p --backend p2p
  run_bench ce --backend ce
  compare_pair nccl_vs_p2p "$OUT/nccl" "$OUT/p2p"
  compare_pair nccl_vs_ce "$OUT/nccl" "$OUT/ce"
fi
REF_BIN="$PWD/baseline/_ref/bin"
if [[ "${CHECK_REFERENCE:-1}" == 1 && "$INIT" == legacy && -x "$REF_BIN/ring_attention_nccl_gpu_bench" ]]; then
  run_reference() {  # label, program
    local dir="$OUT/$1"
    mkdir -p "$dir"
    (cd "$dir" && ATTENTION_DUMP_OUTPUT=1 timeout -k 30 600 python -m torch.distributed.run \
        --nnodes=1 --nproc-per-node "$NP" --master-addr 127.0.0.1 --master-port "$PORT" \
        --no-python "$REF_BIN/$2" "$SIZE" "$WARMUP" "$ITERS" > bench.log 2>&1)
    PORT=$((PORT + 1))
    ./build/bin/verify_full "$dir" "$NP" "$SIZE" | tee "$dir/verify.log" | tail -1
  }
  run_reference reference_nccl ring_attention_nccl_gpu_bench
  run_reference reference_cuda_aware_overlap ring_attention_cuda_aware_Isendrecv_overlap_gpu_bench
  compare_pair nccl_vs_reference_nccl "$OUT/nccl" "$OUT/reference_nccl"
  compare_pair nccl_overlap_vs_reference_overlap "$OUT/nccl_overlap" "$OUT/reference_cuda_aware_overlap"
fi
