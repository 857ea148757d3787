# Standalone native tools (no Python needed to run them):
#   build/bin/rattn_demo           scheduler comparison CLI
#   build/bin/verify_full          full-reference checker for output dumps
# `make cuda-tools` adds the GPU benchmark executables, linked against libtorch,
# NCCL and this tree's sm_100a kernels (launch with `torchrun --no-python`):
#   build/bin/ring_loop_bench      pure ring exchange (p2p | ce | nccl | staged)
#   build/bin/ring_attention_bench ring attention (fused | nccl | staged; fp32 | bf16)
#   build/bin/check_peer           peer-access matrix (the reference's check_peer)
#   build/bin/ring_oneshot         one-shot legacy rings (gpu/ and CPU-attention programs)
# `make mpi-shim` builds build/lib/libmpi_shim.so with csrc/mpi_shim/mpi.h: the
# subset of the MPI C interface the reference prototype's programs call, over a
# TCP store, so they build and run unmodified under torchrun without an MPI.
CXX      ?= g++
NVCC     ?= nvcc
PY       ?= python
CXXFLAGS ?= -O2 -std=c++17 -Wall -Wextra
BIN      := build/bin
OBJ      := build/obj
SCHED    := csrc/sched/workload.cpp csrc/sched/scheduler.cpp csrc/sched/shard_plan.cpp

all: $(BIN)/rattn_demo $(BIN)/verify_full

$(BIN) $(OBJ):
	mkdir -p $@

$(BIN)/rattn_demo: csrc/sched/rattn_demo.cpp $(SCHED) $(wildcard csrc/sched/*.hpp) | $(BIN)
	$(CXX) $(CXXFLAGS) -o $@ csrc/sched/rattn_demo.cpp $(SCHED)

$(BIN)/verify_full: csrc/bench/verify_full.cpp $(SCHED) csrc/common/synth.hpp | $(BIN)
	$(CXX) $(CXXFLAGS) -pthread -o $@ csrc/bench/verify_full.cpp $(SCHED)

# ---------------------------------------------------------------- GPU executables
TORCH_DIR := $(shell $(PY) -c "import os, torch; print(os.path.dirname(torch.__file__))" 2>/dev/null)
NCCL_DIR  := $(shell $(PY) -c "import nvidia.nccl as n; print(list(n.__path__)[0])" 2>/dev/null)
CUDA_HOME ?= /usr/local/cuda
TORCH_INC := -isystem $(TORCH_DIR)/include -isystem $(TORCH_DIR)/include/torch/csrc/api/include \
             -isystem $(NCCL_DIR)/include -isystem $(CUDA_HOME)/include -Icsrc
TORCH_DEF := -D_GLIBCXX_USE_CXX11_ABI=1 $(if $(filter 1,$(MGFA_DEBUG)),-DMGFA_DEBUG)
GPU_CXX   := $(CXX) -O3 -std=c++17 -fPIC -pthread $(TORCH_DEF) $(TORCH_INC)
GPU_NVCC  := $(NVCC) -O3 -std=c++17 -lineinfo --expt-relaxed-constexpr \
             -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC $(TORCH_DEF) $(TORCH_INC) \
             -D__CUDA_NO_HALF_OPERATORS__ -D__CUDA_NO_HALF_CONVERSIONS__ \
             -D__CUDA_NO_BFLOAT16_CONVERSIONS__ -D__CUDA_NO_HALF2_OPERATORS__
GPU_LIBS  := -L$(TORCH_DIR)/lib -Wl,-rpath,$(TORCH_DIR)/lib -ltorch -ltorch_cpu -ltorch_cuda \
             -lc10 -lc10_cuda -L$(NCCL_DIR)/lib -Wl,-rpath,$(NCCL_DIR)/lib -l:libnccl.so.2 \
             -L$(CUDA_HOME)/lib64 -lcudart -pthread
HDRS      := $(wildcard csrc/*/*.hpp csrc/*/*.cuh csrc/*/*.h)

$(OBJ)/%.o: csrc/%.cpp $(HDRS) | $(OBJ)
	@mkdir -p $(dir $@)
	$(GPU_CXX) -c $< -o $@

$(OBJ)/%.o: csrc/%.cu $(HDRS) | $(OBJ)
	@mkdir -p $(dir $@)
	$(GPU_NVCC) -c $< -o $@

SCHED_OBJ := $(OBJ)/sched/workload.o $(OBJ)/sched/scheduler.o $(OBJ)/sched/shard_plan.o
COMM_OBJ  := $(OBJ)/bench/dist_env.o $(OBJ)/mpi_shim/mpi_shim.o $(OBJ)/comm/symmetric.o \
             $(OBJ)/kernels/ring_exchange.o

$(BIN)/ring_loop_bench: $(OBJ)/bench/ring_loop_bench.o $(COMM_OBJ) | $(BIN)
	$(CXX) -o $@ $^ $(GPU_LIBS)

$(BIN)/ring_attention_bench: $(OBJ)/bench/ring_attention_bench.o $(COMM_OBJ) $(SCHED_OBJ) \
    $(OBJ)/kernels/flash_fwd_sm100.o $(OBJ)/kernels/flash_bwd_sm100.o $(OBJ)/kernels/legacy_fp32.o \
    $(OBJ)/kernels/attn_fwd_persistent.o $(OBJ)/ops/attn_api.o | $(BIN)
	$(CXX) -o $@ $^ $(GPU_LIBS)

$(BIN)/ring_oneshot: $(OBJ)/bench/ring_oneshot.o $(COMM_OBJ) $(OBJ)/kernels/legacy_fp32.o \
    $(OBJ)/host/cpu_attention.o | $(BIN)
	$(CXX) -o $@ $^ $(GPU_LIBS)

$(BIN)/check_peer: csrc/bench/check_peer.cpp | $(BIN)
	$(CXX) -O2 -std=c++17 -isystem $(CUDA_HOME)/include -o $@ $< -L$(CUDA_HOME)/lib64 -Wl,-rpath,$(CUDA_HOME)/lib64 -lcudart

$(BIN)/dist_selftest: $(OBJ)/bench/dist_selftest.o $(OBJ)/bench/dist_env.o \
    $(OBJ)/mpi_shim/mpi_shim.o | $(BIN)
	$(CXX) -o $@ $^ $(GPU_LIBS)

LIB := build/lib
$(LIB)/libmpi_shim.so: csrc/mpi_shim/mpi_shim.cpp csrc/mpi_shim/mpi.h
	@mkdir -p $(LIB)
	$(GPU_CXX) -Icsrc/mpi_shim -shared -o $@ $< -L$(TORCH_DIR)/lib -Wl,-rpath,$(TORCH_DIR)/lib \
	    -ltorch_cpu -lc10 -L$(CUDA_HOME)/lib64 -Wl,-rpath,$(CUDA_HOME)/lib64 -lcudart

mpi-shim: $(LIB)/libmpi_shim.so

cuda-tools: $(BIN)/ring_loop_bench $(BIN)/ring_attention_bench $(BIN)/check_peer \
    $(BIN)/dist_selftest $(BIN)/ring_oneshot

clean:
	rm -rf $(BIN) $(OBJ) $(LIB)

.PHONY: all cuda-tools mpi-shim clean
