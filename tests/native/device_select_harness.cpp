// Differential-test harness for the local-rank and device binding rules
// (csrc/common/device_select.hpp) against the reference prototype's own
// read_local_rank_from_env / select_local_cuda_device (its
// ring/attention/common/device_utils.cuh, included as written, REF_HEADER).
// The CUDA device count comes from a stand-in cudaGetDeviceCount defined here
// (argument <count>), so no GPU is needed; MPI is this repository's subset.
//   device_select_harness ref|ours <count>
//   -> "local <L> device <D>", or exit status 1 where the binding is refused
#include <cuda_runtime_api.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

static int g_count = 0;
extern "C" cudaError_t cudaGetDeviceCount(int* count) {
  *count = g_count;
  return cudaSuccess;
}
extern "C" cudaError_t cudaSetDevice(int) { return cudaSuccess; }
extern "C" const char* cudaGetErrorString(cudaError_t) { return "stand-in"; }

#include REF_HEADER

#include "common/device_select.hpp"

int main(int argc, char** argv) {
  if (argc < 3) return 2;
  g_count = std::atoi(argv[2]);
  if (std::strcmp(argv[1], "ref") == 0) {
    MPI_Init(&argc, &argv);
    int local = -1;
    const int dev = select_local_cuda_device(MPI_COMM_WORLD, 0, &local);
    std::printf("local %d device %d\n", local, dev);
    MPI_Finalize();
    return 0;
  }
  // rank 0 of a one-process job: the reference's shared-memory split gives 0
  const mgfa::DeviceChoice c = mgfa::choose_device(g_count, 0);
  if (!c.error.empty()) {
    std::fprintf(stderr, "%s\n", c.error.c_str());
    return 1;
  }
  std::printf("local %d device %d\n", c.local_rank, c.device);
  return 0;
}
