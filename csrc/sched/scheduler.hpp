// Static partitioners over the attention workload model.
//
// Parity with the reference prototype (workload/scheduler.c):
//   * round-robin: task t -> gpu t % G                   -- scheduler.c:27-41
//   * block LPT: cost-descending order, each task to the least-loaded gpu
//     (lowest id among ties)                             -- scheduler.c:86-134
//   * single best move / best swap off the heaviest gpu  -- scheduler.c:137-251
//   * row-level LPT with RowTask::total_cost as the unit -- scheduler.c:254-281
//   * contiguous-row DP: dp[g][i] = min_k max(dp[g-1][k], prefix[i]-prefix[k]),
//     -1 when G > rows                                   -- scheduler.c:284-356
// Differences, on purpose:
//   * LPT sorts with std::stable_sort, so ties keep task order and the
//     assignment is deterministic on every libc (the reference's qsort order for
//     equal costs is libc-specific; loads and makespans are the same either way).
//   * LptMode::Heap is a real O(T log G) heap keyed on (load, gpu id), which
//     picks the same gpu as the linear scan; Auto uses it for G >= 16.
//   * rebalance_swap_once considers every task as a partner. The reference
//     indexes task_to_gpu with a gpu-range loop variable (scheduler.c:211-212),
//     so only tasks 0..G-1 are partners; `reference_partner_quirk=true` keeps
//     that behaviour for comparisons.
//   * the DP uses heap storage (the reference uses stack VLAs).
#pragma once

#include <vector>

#include "workload.hpp"

namespace mgfa::sched {

enum class LptMode : int { Scan = 0, Heap = 1, Auto = 2 };

struct GpuLoad {
  int gpu = 0;
  int task_count = 0;
  double total_cost = 0.0;
};

struct Assignment {
  std::vector<GpuLoad> gpus;     // one entry per gpu
  std::vector<int> task_to_gpu;  // -1 = unassigned
  double makespan() const;
  int most_loaded() const;   // first gpu with the largest load
  int least_loaded() const;  // first gpu with the smallest load
};

Assignment empty_assignment(int num_gpus, int num_tasks);

Assignment assign_round_robin(const std::vector<BlockTask>& tasks, int num_gpus);
Assignment assign_lpt(const std::vector<double>& costs, int num_gpus,
                      LptMode mode = LptMode::Scan);
Assignment assign_block_lpt(const std::vector<BlockTask>& tasks, int num_gpus,
                            LptMode mode = LptMode::Scan);
Assignment assign_row_lpt(const std::vector<RowTask>& rows, int num_gpus,
                          LptMode mode = LptMode::Scan);

// Apply the single move (or swap) that lowers the makespan most; false when none
// lowers it.
bool rebalance_move_once(const std::vector<double>& costs, Assignment* a);
bool rebalance_swap_once(const std::vector<double>& costs, Assignment* a,
                         bool reference_partner_quirk = false);

struct RowShard {
  int gpu = 0;
  int row_begin = 0;  // [row_begin, row_end)
  int row_end = 0;
  double total_cost = 0.0;
};

struct ContiguousPartition {
  bool ok = false;  // false when num_gpus > rows or inputs are empty
  std::vector<RowShard> shards;
  std::vector<int> row_to_gpu;
  double makespan() const;
};

ContiguousPartition partition_rows_contiguous(const std::vector<RowTask>& rows,
                                              int num_gpus);

std::vector<double> task_costs(const std::vector<BlockTask>& tasks);
std::vector<double> row_costs(const std::vector<RowTask>& rows);

}  // namespace mgfa::sched
