// rattn_demo: compare static partitions of one attention workload.
//
//   rattn_demo --seq N --gpus G [--block B] [--mask causal|full] [--alpha a]
//              [--beta b] [--report] [--max-tasks T] [--max-rows R]
//
// Without --report it prints the one fixed-width table row of the reference
// demo (workload/demo.c:108-118): seq, gpus, mask, blocks, then makespan and
// imbalance for round-robin, block LPT, row LPT and contiguous DP, then the
// ideal makespan. Conventions kept from the reference (workload/demo.c:14-124):
//   * defaults block 128, alpha 1.21, beta 3.84e-6, causal;
//   * tasks are costed with alpha = 0 and alpha is added once to every makespan;
//   * imbalance = makespan / ideal, ideal = alpha + total / G;
//   * at most 4096 block tasks (later blocks are left out, as there) and 256
//     block rows (beyond that the row partitions are skipped and the row shows
//     what the reference's shows then: alpha alone for row LPT, N/A for DP);
//     --max-tasks / --max-rows lift those caps;
//   * only "--mask full" changes the mask, any other word leaves it as it was.
// --report adds per-gpu loads and max/mean imbalance for every partition and,
// for the row partitions, the step-paced imbalance of a ring whose ranks own
// those rows (each ring step advances at its slowest rank's pace).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "scheduler.hpp"
#include "shard_plan.hpp"
#include "workload.hpp"

using namespace mgfa::sched;

static void usage(const char* prog) {
  std::printf(
      "Usage: %s --seq <N> --gpus <G> [--block <B>] [--mask causal|full] [--alpha <a>] "
      "[--beta <b>]\n",
      prog);
}

static void print_loads(const char* name, const std::vector<double>& loads, double alpha) {
  double mx = 0.0, sum = 0.0;
  for (double l : loads) { mx = l > mx ? l : mx; sum += l; }
  const double mean = loads.empty() ? 0.0 : sum / double(loads.size());
  std::printf("  %-8s max/mean=%.4f loads:", name, mean > 0 ? mx / mean : 1.0);
  for (double l : loads) std::printf(" %.4f", alpha + l);
  std::printf("\n");
}

// Sum over the ring's steps of the slowest rank's visible pairs, over the mean
// per-rank total, when rank g owns the block rows with row_to_gpu[row] == g.
static double ring_paced(int seq, int block, const std::vector<int>& row_to_gpu, int world,
                         MaskKind mask) {
  const ShardPlan plan = make_from_rows(seq, block, row_to_gpu, world);
  double paced = 0.0, total = 0.0;
  for (int t = 0; t < world; ++t) {
    double slowest = 0.0;
    for (int r = 0; r < world; ++r) {
      const double w = double(step_active(plan, r, plan.compute_owner(r, t), mask));
      slowest = w > slowest ? w : slowest;
      total += w;
    }
    paced += slowest;
  }
  return total > 0.0 ? paced / (total / world) : 1.0;
}

int main(int argc, char** argv) {
  int seq = 0, gpus = 0, block = 128;
  MaskKind mask = MaskKind::Causal;
  double alpha = 1.21, beta = 0.00000384;
  bool report = false;
  long long max_tasks = 4096, max_rows = 256;

  for (int i = 1; i < argc; ++i) {
    const bool has_val = i + 1 < argc;
    if (!std::strcmp(argv[i], "--seq") && has_val) seq = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--gpus") && has_val) gpus = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--block") && has_val) block = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--mask") && has_val) {
      ++i;
      if (!std::strcmp(argv[i], "full")) mask = MaskKind::Full;
    } else if (!std::strcmp(argv[i], "--alpha") && has_val) alpha = std::atof(argv[++i]);
    else if (!std::strcmp(argv[i], "--beta") && has_val) beta = std::atof(argv[++i]);
    else if (!std::strcmp(argv[i], "--max-tasks") && has_val) max_tasks = std::atoll(argv[++i]);
    else if (!std::strcmp(argv[i], "--max-rows") && has_val) max_rows = std::atoll(argv[++i]);
    else if (!std::strcmp(argv[i], "--report")) report = true;
  }
  if (seq <= 0 || gpus <= 0 || block <= 0) {
    usage(argv[0]);
    return 1;
  }

  const WorkloadShape shape{seq, seq, block, block};
  const CostModel task_model{0.0, beta};
  std::vector<BlockTask> tasks =
      build_block_tasks(shape, mask, task_model, size_t(max_tasks < 0 ? 0 : max_tasks));
  const int count = int(tasks.size());

  double total = 0.0;
  for (const BlockTask& t : tasks) total += t.cost;
  const double ideal = alpha + total / gpus;

  Assignment rr = assign_round_robin(tasks, gpus);
  const double rr_ms = alpha + rr.makespan();
  Assignment blk = assign_block_lpt(tasks, gpus, LptMode::Scan);
  const double blk_ms = alpha + blk.makespan();

  // More block rows than the row cap: the reference demo then assigns no rows
  // (its row builder fails and the row LPT runs over none), so its table shows
  // alpha alone for row LPT and N/A for DP. The table row is kept the same; a
  // warning on stderr says that the row partitions were skipped.
  const bool rows_fit = num_row_blocks(shape) <= max_rows;
  if (!rows_fit)
    std::fprintf(stderr,
                 "warning: %d block rows exceed --max-rows %lld; the row partitions are "
                 "skipped (row LPT shows alpha alone, DP N/A)\n",
                 num_row_blocks(shape), max_rows);
  std::vector<RowTask> rows = rows_fit ? build_row_tasks(shape, tasks) : std::vector<RowTask>{};
  Assignment row = assign_row_lpt(rows, gpus, LptMode::Scan);
  const double row_ms = alpha + row.makespan();

  ContiguousPartition dp = partition_rows_contiguous(rows, gpus);
  const double dp_ms = dp.ok ? alpha + dp.makespan() : -1.0;

  std::printf("%-6d %-5d %-6s %-6d | %-10.2f %-6.3f | %-10.2f %-6.3f | %-10.2f %-6.3f | ", seq,
              gpus, mask_name(mask), count, rr_ms, rr_ms / ideal, blk_ms, blk_ms / ideal, row_ms,
              row_ms / ideal);
  if (dp_ms >= 0) std::printf("%-10.2f %-6.3f | ", dp_ms, dp_ms / ideal);
  else std::printf("%-10s %-6s | ", "N/A", "N/A");
  std::printf("%-10.2f\n", ideal);

  if (report) {
    std::printf("per-gpu loads (alpha added once per gpu):\n");
    auto loads_of = [](const Assignment& a) {
      std::vector<double> v;
      for (const GpuLoad& g : a.gpus) v.push_back(g.total_cost);
      return v;
    };
    print_loads("RR", loads_of(rr), alpha);
    print_loads("BlkLPT", loads_of(blk), alpha);
    print_loads("RowLPT", loads_of(row), alpha);
    if (dp.ok) {
      std::vector<double> v;
      for (const RowShard& s : dp.shards) v.push_back(s.total_cost);
      print_loads("DP", v, alpha);
      std::printf("  DP shards (block rows):");
      for (const RowShard& s : dp.shards) std::printf(" [%d,%d)", s.row_begin, s.row_end);
      std::printf("\n");
    }
    const bool truncated = max_tasks > 0 && tasks.size() >= size_t(max_tasks);
    if (!rows_fit) {
      std::printf("row partitions: skipped (%d block rows exceed --max-rows %lld)\n",
                  num_row_blocks(shape), max_rows);
    } else if (truncated) {
      std::printf("ring step-paced imbalance: n/a (block tasks truncated at --max-tasks)\n");
    } else if (int(rows.size()) == num_row_blocks(shape)) {
      std::vector<int> r2g(rows.size(), 0);
      for (size_t i = 0; i < rows.size(); ++i) r2g[size_t(rows[i].row)] = row.task_to_gpu[i];
      std::printf("ring step-paced imbalance: RowLPT=%.3f", ring_paced(seq, block, r2g, gpus, mask));
      if (dp.ok) {
        std::vector<int> d2g(rows.size(), 0);
        for (size_t g = 0; g < dp.shards.size(); ++g)
          for (int rr = dp.shards[g].row_begin; rr < dp.shards[g].row_end; ++rr) d2g[size_t(rr)] = int(g);
        std::printf(" DP=%.3f", ring_paced(seq, block, d2g, gpus, mask));
      }
      std::printf("\n");
    }
    std::printf("block rows:");
    for (const RowTask& r : rows)
      std::printf(" %d:%d/%d", r.row, r.num_blocks, r.num_cols_needed);
    std::printf("\n");
  }
  return 0;
}
