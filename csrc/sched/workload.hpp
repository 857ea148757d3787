// Attention workload model: block grid, masks, active-element counts and a
// linear cost model.
//
// Parity with the reference prototype (Multi-GPU-Flashattention):
//   * mask rule "key k visible to query q iff k <= q" for causal, all-visible for
//     full                                        -- workload/workload.c:20-28
//   * block grid = ceil(seq / block) per axis     -- workload/workload.c:7-17
//   * cost = alpha + beta * active, 0 when empty  -- workload/workload.c:45-51
//   * only non-empty blocks become tasks          -- workload/workload.c:54-97
//   * row aggregation (num_blocks, rightmost col + 1, summed cost, comm = 0)
//                                                 -- workload/workload.c:100-137
// The active count is computed in closed form (O(rows) per block instead of the
// reference's O(block_q * block_k) brute force); `count_active_bruteforce`
// keeps the brute-force definition for tests.
#pragma once

#include <cstddef>
#include <cstdint>
#include <limits>
#include <string>
#include <vector>

namespace mgfa::sched {

enum class MaskKind : int { Causal = 0, Full = 1 };

const char* mask_name(MaskKind m);
bool parse_mask(const std::string& s, MaskKind* out);

struct WorkloadShape {
  int seq_q = 0;
  int seq_k = 0;
  int block_q = 128;
  int block_k = 128;
};

struct CostModel {
  double alpha = 0.0;  // fixed cost per non-empty task
  double beta = 0.0;   // cost per active (unmasked) score element
};

struct BlockTask {
  int row = 0;
  int col = 0;
  int q_begin = 0, q_end = 0;  // [begin, end) token ranges
  int k_begin = 0, k_end = 0;
  int64_t active = 0;
  int64_t total = 0;
  double cost = 0.0;
  double density = 0.0;
};

struct RowTask {
  int row = 0;
  int num_blocks = 0;
  int num_cols_needed = 0;  // rightmost non-empty block column + 1
  double comp_cost = 0.0;
  double comm_cost = 0.0;   // not modelled yet: always 0
  double total_cost = 0.0;
};

int num_row_blocks(const WorkloadShape& s);
int num_col_blocks(const WorkloadShape& s);
int64_t total_blocks(const WorkloadShape& s);

// 1 if key position k is visible to query position q under `m`.
inline int mask_value(MaskKind m, int64_t q, int64_t k) {
  return m == MaskKind::Full ? 1 : (k <= q ? 1 : 0);
}

// Number of visible (q, k) pairs in [q_begin, q_end) x [k_begin, k_end).
int64_t count_active(MaskKind m, int64_t q_begin, int64_t q_end, int64_t k_begin,
                     int64_t k_end);
int64_t count_active_bruteforce(MaskKind m, int64_t q_begin, int64_t q_end,
                                int64_t k_begin, int64_t k_end);

double estimate_cost(const CostModel& model, int64_t active);

// All non-empty blocks in row-major order, at most `max_tasks` of them (the
// list is cut short, silently, once it is full -- the reference behaves the same
// way and its demo relies on a 4096 cap).
std::vector<BlockTask> build_block_tasks(
    const WorkloadShape& s, MaskKind m, const CostModel& model,
    size_t max_tasks = std::numeric_limits<size_t>::max());

// One RowTask per block row of the grid (rows with no task have zero cost).
std::vector<RowTask> build_row_tasks(const WorkloadShape& s,
                                     const std::vector<BlockTask>& tasks);

}  // namespace mgfa::sched
