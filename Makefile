# Standalone native tools (no Python needed):
#   build/bin/rattn_demo     scheduler comparison CLI
#   build/bin/verify_full    full-reference checker for output dumps
# `make cuda-tools` adds the GPU benchmarks (see csrc/bench).
CXX      ?= g++
NVCC     ?= nvcc
CXXFLAGS ?= -O2 -std=c++17 -Wall -Wextra
BIN      := build/bin
SCHED    := csrc/sched/workload.cpp csrc/sched/scheduler.cpp csrc/sched/shard_plan.cpp

all: $(BIN)/rattn_demo $(BIN)/verify_full

$(BIN):
	mkdir -p $(BIN)

$(BIN)/rattn_demo: csrc/sched/rattn_demo.cpp $(SCHED) $(wildcard csrc/sched/*.hpp) | $(BIN)
	$(CXX) $(CXXFLAGS) -o $@ csrc/sched/rattn_demo.cpp $(SCHED)

$(BIN)/verify_full: csrc/bench/verify_full.cpp $(SCHED) csrc/common/synth.hpp | $(BIN)
	$(CXX) $(CXXFLAGS) -pthread -o $@ csrc/bench/verify_full.cpp $(SCHED)

clean:
	rm -rf $(BIN)

.PHONY: all clean
