#!/usr/bin/env bash
# Builds the reference prototype's programs, unmodified, into baseline/_ref/bin:
# the workload demo, the MPI ring test, the ring-exchange loops and the ring
# attention benchmarks (staged MPI, CUDA-aware MPI, NCCL), plus verify_full.
# MPI comes from this repository's libmpi_shim (csrc/mpi_shim, `make mpi-shim`),
# so the programs run under `torchrun --no-python` with no MPI installation;
# CUDA code is compiled for sm_100a. The reference tree is read from REF_SRC.
#
#   benchmarks/build_reference.sh            # build everything
#   benchmarks/build_reference.sh --cpu-only # rattn_demo, verify_full, ring_test
#   benchmarks/build_reference.sh --print-src # where the reference tree is read from
#   REF_SRC=/path/to/reference OUT=dir benchmarks/build_reference.sh
# Exit status 2: no reference tree at REF_SRC.
set -euo pipefail
cd "$(dirname "$0")/.."
REF=${REF_SRC:-/root/reference}
OUT=${OUT:-baseline/_ref}
PY=${PY:-python}
NVCC=${NVCC:-nvcc}
CUDA_HOME=${CUDA_HOME:-/usr/local/cuda}
[ -d "$REF/ring" ] || { echo "reference tree not found at $REF" >&2; exit 2; }
if [ "${1:-}" = "--print-src" ]; then echo "$REF"; exit 0; fi

make -s mpi-shim
SHIM_INC="$PWD/csrc/mpi_shim"
SHIM_LIB="$PWD/build/lib"
NCCL_DIR=$($PY -c "import nvidia.nccl as n; print(list(n.__path__)[0])")
MPI_FLAGS=(-I"$SHIM_INC" -L"$SHIM_LIB" -Xlinker -rpath -Xlinker "$SHIM_LIB" -lmpi_shim)
NCCL_FLAGS=(-I"$NCCL_DIR/include" -L"$NCCL_DIR/lib" -Xlinker -rpath -Xlinker "$NCCL_DIR/lib" -l:libnccl.so.2)
ARCH=(-gencode arch=compute_100a,code=sm_100a)
mkdir -p "$OUT/bin"
BIN=$(cd "$OUT/bin" && pwd)

cc_c() {   # name sources... (flags as the reference's own build lines: -O2)
  local name=$1; shift
  echo "  gcc  $name"
  gcc -O2 -o "$BIN/$name" "$@" -lm
}
cc_cu() {  # name source [extra flags]
  local name=$1 src=$2; shift 2
  echo "  nvcc $name"
  "$NVCC" -O3 "${ARCH[@]}" -o "$BIN/$name" "$src" "${MPI_FLAGS[@]}" "$@"
}

echo "building the reference from $REF into $OUT/bin"
# CPU programs
cc_c rattn_demo -std=c11 "$REF/workload/demo.c" "$REF/workload/workload.c" "$REF/workload/scheduler.c" -I"$REF/workload"
cc_c verify_full "$REF/ring/attention/verify_full.c"
cc_c ring_test "$REF/ring/ring_test.c" -I"$SHIM_INC" -L"$SHIM_LIB" -Wl,-rpath,"$SHIM_LIB" -lmpi_shim
if [ "${1:-}" = "--cpu-only" ]; then
  echo "done: CPU programs in $OUT/bin"
  exit 0
fi
# ring basics
cc_cu check_peer "$REF/ring/check_peer.cu"
cc_cu ring_cuda "$REF/ring/ring_cuda.cu"
# pure ring-exchange loops
for f in ring_loop_staged ring_loop_staged_Isendrecv ring_loop_cuda_aware ring_loop_cuda_aware_Isendrecv; do
  cc_cu "$f" "$REF/ring/loop/$f.cu"
done
cc_cu ring_loop_nccl "$REF/ring/loop/ring_loop_nccl.cu" "${NCCL_FLAGS[@]}"
# ring attention: CPU-math variants, GPU variants, benchmark variants
for f in ring_attention_staged ring_attention_cuda_aware; do
  cc_cu "$f" "$REF/ring/attention/$f.cu"
done
for f in ring_attention_staged_gpu ring_attention_cuda_aware_gpu; do
  cc_cu "$f" "$REF/ring/attention/gpu/$f.cu"
done
cc_cu ring_attention_nccl_gpu "$REF/ring/attention/gpu/ring_attention_nccl_gpu.cu" "${NCCL_FLAGS[@]}"
for f in ring_attention_staged_gpu_bench ring_attention_staged_Isendrecv_gpu_bench \
         ring_attention_staged_Isendrecv_overlap_gpu_bench ring_attention_cuda_aware_gpu_bench \
         ring_attention_cuda_aware_Isendrecv_gpu_bench ring_attention_cuda_aware_Isendrecv_overlap_gpu_bench; do
  cc_cu "$f" "$REF/ring/attention/bench/$f.cu"
done
cc_cu ring_attention_nccl_gpu_bench "$REF/ring/attention/bench/ring_attention_nccl_gpu_bench.cu" "${NCCL_FLAGS[@]}"
echo "done: $(ls "$BIN" | wc -l) programs in $OUT/bin"
