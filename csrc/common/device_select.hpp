// Local-rank -> CUDA device binding for one-process-per-GPU launches.
//
// Local rank comes from the first set variable of OMPI_COMM_WORLD_LOCAL_RANK,
// MV2_COMM_WORLD_LOCAL_RANK, SLURM_LOCALID, MPI_LOCALRANKID, PMI_LOCAL_RANK,
// PALS_LOCAL_RANK (the launcher list of the reference's
// ring/attention/common/device_utils.cuh:9-27) and then LOCAL_RANK (torchrun).
// Without any of them the caller supplies a fallback (e.g. the rank within the
// node from its process group). More ranks than devices is refused unless
// ALLOW_GPU_OVERSUBSCRIBE is set, in which case device = local_rank % count
// (device_utils.cuh:43-79).
#pragma once

#include <cstdlib>
#include <string>

namespace mgfa {

inline const char* const kLocalRankVars[] = {
    "OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK", "SLURM_LOCALID",
    "MPI_LOCALRANKID",            "PMI_LOCAL_RANK",            "PALS_LOCAL_RANK",
    "LOCAL_RANK"};

// Local rank from the environment, or -1 when none of the variables is set.
inline int local_rank_from_env(std::string* source = nullptr) {
  for (const char* name : kLocalRankVars) {
    const char* v = std::getenv(name);
    if (v && v[0] != '\0') {
      if (source) *source = name;
      return std::atoi(v);
    }
  }
  return -1;
}

struct DeviceChoice {
  int device = -1;       // -1 on error
  int local_rank = -1;
  std::string source;    // which variable (or "fallback")
  std::string error;     // non-empty on error
};

inline DeviceChoice choose_device(int device_count, int fallback_local_rank) {
  DeviceChoice c;
  c.local_rank = local_rank_from_env(&c.source);
  if (c.local_rank < 0) {
    c.local_rank = fallback_local_rank;
    c.source = "fallback";
  }
  if (device_count <= 0) {
    c.error = "No CUDA devices found.";
    return c;
  }
  const bool oversubscribe = std::getenv("ALLOW_GPU_OVERSUBSCRIBE") != nullptr;
  if (c.local_rank >= device_count && !oversubscribe) {
    c.error = "local_rank " + std::to_string(c.local_rank) + ": only " +
              std::to_string(device_count) +
              " CUDA device(s) are visible. Reduce ranks per node or set "
              "ALLOW_GPU_OVERSUBSCRIBE=1.";
    return c;
  }
  c.device = c.local_rank % device_count;
  return c;
}

}  // namespace mgfa
