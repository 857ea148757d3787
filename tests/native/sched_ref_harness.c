/* Differential-test harness for the workload model and schedulers: built by
 * tests/test_reference_live_cpu.py against the reference prototype's
 * workload/workload.c and workload/scheduler.c (its public functions, declared
 * in its workload.h and scheduler.h), it prints every intermediate result for
 * one workload, so the test can compare them line by line with this
 * repository's C++ implementation (through the _sched bindings).
 *
 *   sched_ref_harness <seq> <block> <gpus> <causal 0|1> <alpha> <beta>
 *
 * Output (one record per line, doubles with 17 significant digits):
 *   T row col q_begin q_end k_begin k_end active total cost density
 *   RR gpu... | LPT_SCAN gpu... | LPT_HEAP gpu... | LPT_AUTO gpu...  task -> gpu maps
 *   MOVE moved gpu...        one move repair applied to the round-robin map
 *   SWAP swapped gpu...      one swap repair applied to the round-robin map
 *                            ("SWAP n/a" with more gpus than tasks: the
 *                            reference's swap then reads past its task array)
 *   R row num_blocks num_cols_needed comp_cost total_cost
 *   ROWLPT gpu...            row -> gpu
 *   DP status gpu...         row -> gpu of the contiguous partition */
#include <stdio.h>
#include <stdlib.h>

#include "scheduler.h"
#include "workload.h"

static void print_map(const char* tag, const int* map, int n) {
  printf("%s", tag);
  for (int i = 0; i < n; ++i) printf(" %d", map[i]);
  printf("\n");
}

int main(int argc, char** argv) {
  if (argc < 7) return 2;
  const int seq = atoi(argv[1]), block = atoi(argv[2]), gpus = atoi(argv[3]);
  struct workload_input op = {seq, seq, block, block};
  struct mask_desc mask = {atoi(argv[4]) ? MASK_CAUSAL : MASK_FULL};
  struct cost_model model = {atof(argv[5]), atof(argv[6])};
  enum { kMaxTasks = 4096, kMaxRows = 256 };
  struct block_task* tasks = malloc(kMaxTasks * sizeof(*tasks));
  const int n = build_tasks(&op, &mask, &model, tasks, kMaxTasks);
  for (int t = 0; t < n; ++t)
    printf("T %d %d %d %d %d %d %d %d %.17g %.17g\n", tasks[t].row_idx, tasks[t].col_idx,
           tasks[t].q_begin, tasks[t].q_end, tasks[t].k_begin, tasks[t].k_end, tasks[t].active,
           tasks[t].total, tasks[t].cost, tasks[t].density);
  struct gpu_load* loads = malloc(gpus * sizeof(*loads));
  int* map = malloc((n > 0 ? n : 1) * sizeof(int));
  assign_round_robin(tasks, n, loads, gpus, map);
  print_map("RR", map, n);
  int moved = rebalance_move_once(tasks, n, loads, gpus, map);
  printf("MOVE %d", moved);
  print_map("", map, n);
  if (gpus <= n) {  /* its partner loop indexes the task array by gpu: needs gpus <= tasks */
    assign_round_robin(tasks, n, loads, gpus, map);
    int swapped = rebalance_swap_once(tasks, n, loads, gpus, map);
    printf("SWAP %d", swapped);
    print_map("", map, n);
  } else {
    printf("SWAP n/a\n");
  }
  assign_lpt(tasks, n, loads, gpus, map, LPT_SCAN);
  print_map("LPT_SCAN", map, n);
  assign_lpt(tasks, n, loads, gpus, map, LPT_HEAP);
  print_map("LPT_HEAP", map, n);
  assign_lpt(tasks, n, loads, gpus, map, LPT_AUTO);
  print_map("LPT_AUTO", map, n);
  struct row_task* rows = malloc(kMaxRows * sizeof(*rows));
  const int nr = build_row_tasks(&op, tasks, n, rows, kMaxRows);
  if (nr > 0) {
    for (int r = 0; r < nr; ++r)
      printf("R %d %d %d %.17g %.17g\n", rows[r].row_idx, rows[r].num_blocks,
             rows[r].num_cols_needed, rows[r].comp_cost, rows[r].total_cost);
    int* rmap = malloc(nr * sizeof(int));
    assign_row_tasks_lpt(rows, nr, loads, gpus, rmap);
    print_map("ROWLPT", rmap, nr);
    struct row_shard* shards = malloc(gpus * sizeof(*shards));
    const int st = partition_rows_contiguous(rows, nr, shards, gpus, rmap);
    printf("DP %d", st);
    print_map("", rmap, st == 0 ? nr : 0);
    free(shards);
    free(rmap);
  }
  free(rows);
  free(map);
  free(loads);
  free(tasks);
  return 0;
}
