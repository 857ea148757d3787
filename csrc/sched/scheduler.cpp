#include "scheduler.hpp"

#include <algorithm>
#include <cfloat>
#include <numeric>
#include <queue>
#include <tuple>

namespace mgfa::sched {

double Assignment::makespan() const {
  double m = 0.0;
  for (const GpuLoad& g : gpus) m = std::max(m, g.total_cost);
  return m;
}

int Assignment::most_loaded() const {
  int best = 0;
  for (int i = 1; i < int(gpus.size()); ++i)
    if (gpus[i].total_cost > gpus[best].total_cost) best = i;
  return best;
}

int Assignment::least_loaded() const {
  int best = 0;
  for (int i = 1; i < int(gpus.size()); ++i)
    if (gpus[i].total_cost < gpus[best].total_cost) best = i;
  return best;
}

Assignment empty_assignment(int num_gpus, int num_tasks) {
  Assignment a;
  a.gpus.resize(std::max(num_gpus, 0));
  for (int i = 0; i < int(a.gpus.size()); ++i) a.gpus[i].gpu = i;
  a.task_to_gpu.assign(std::max(num_tasks, 0), -1);
  return a;
}

std::vector<double> task_costs(const std::vector<BlockTask>& tasks) {
  std::vector<double> c(tasks.size());
  for (size_t i = 0; i < tasks.size(); ++i) c[i] = tasks[i].cost;
  return c;
}

std::vector<double> row_costs(const std::vector<RowTask>& rows) {
  std::vector<double> c(rows.size());
  for (size_t i = 0; i < rows.size(); ++i) c[i] = rows[i].total_cost;
  return c;
}

Assignment assign_round_robin(const std::vector<BlockTask>& tasks, int num_gpus) {
  Assignment a = empty_assignment(num_gpus, int(tasks.size()));
  if (num_gpus <= 0) return a;
  for (int t = 0; t < int(tasks.size()); ++t) {
    const int g = t % num_gpus;
    a.gpus[g].task_count += 1;
    a.gpus[g].total_cost += tasks[t].cost;
    a.task_to_gpu[t] = g;
  }
  return a;
}

Assignment assign_lpt(const std::vector<double>& costs, int num_gpus, LptMode mode) {
  Assignment a = empty_assignment(num_gpus, int(costs.size()));
  if (num_gpus <= 0) return a;
  std::vector<int> order(costs.size());
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int x, int y) { return costs[x] > costs[y]; });

  const bool use_heap = mode == LptMode::Heap || (mode == LptMode::Auto && num_gpus >= 16);
  if (!use_heap) {
    for (int idx : order) {
      const int g = a.least_loaded();
      a.gpus[g].task_count += 1;
      a.gpus[g].total_cost += costs[idx];
      a.task_to_gpu[idx] = g;
    }
    return a;
  }
  // Min-heap on (load, gpu id): the top is the gpu the linear scan would pick.
  using Entry = std::pair<double, int>;
  std::priority_queue<Entry, std::vector<Entry>, std::greater<Entry>> heap;
  for (int g = 0; g < num_gpus; ++g) heap.emplace(0.0, g);
  for (int idx : order) {
    const int g = heap.top().second;
    heap.pop();
    a.gpus[g].task_count += 1;
    a.gpus[g].total_cost += costs[idx];
    a.task_to_gpu[idx] = g;
    heap.emplace(a.gpus[g].total_cost, g);
  }
  return a;
}

Assignment assign_block_lpt(const std::vector<BlockTask>& tasks, int num_gpus, LptMode mode) {
  return assign_lpt(task_costs(tasks), num_gpus, mode);
}

Assignment assign_row_lpt(const std::vector<RowTask>& rows, int num_gpus, LptMode mode) {
  return assign_lpt(row_costs(rows), num_gpus, mode);
}

bool rebalance_move_once(const std::vector<double>& costs, Assignment* a) {
  const int G = int(a->gpus.size());
  if (G < 2) return false;
  const int heavy = a->most_loaded();
  double best = a->makespan();
  int best_task = -1, best_dst = -1;
  for (int t = 0; t < int(costs.size()); ++t) {
    if (a->task_to_gpu[t] != heavy) continue;
    for (int dst = 0; dst < G; ++dst) {
      if (dst == heavy) continue;
      double span = 0.0;
      for (int g = 0; g < G; ++g) {
        double load = a->gpus[g].total_cost;
        if (g == heavy) load -= costs[t];
        else if (g == dst) load += costs[t];
        span = std::max(span, load);
      }
      if (span < best) { best = span; best_task = t; best_dst = dst; }
    }
  }
  if (best_task < 0) return false;
  a->gpus[heavy].task_count -= 1;
  a->gpus[heavy].total_cost -= costs[best_task];
  a->gpus[best_dst].task_count += 1;
  a->gpus[best_dst].total_cost += costs[best_task];
  a->task_to_gpu[best_task] = best_dst;
  return true;
}

bool rebalance_swap_once(const std::vector<double>& costs, Assignment* a,
                         bool reference_partner_quirk) {
  const int G = int(a->gpus.size());
  const int T = int(costs.size());
  if (G < 2) return false;
  const int heavy = a->most_loaded();
  double best = a->makespan();
  int best_task = -1, best_partner = -1;
  const int partners = reference_partner_quirk ? std::min(G, T) : T;
  for (int t = 0; t < T; ++t) {
    if (a->task_to_gpu[t] != heavy) continue;
    for (int p = 0; p < partners; ++p) {
      const int gp = a->task_to_gpu[p];
      if (gp == heavy || gp < 0) continue;
      double span = 0.0;
      for (int g = 0; g < G; ++g) {
        double load = a->gpus[g].total_cost;
        if (g == heavy) load = load - costs[t] + costs[p];
        else if (g == gp) load = load - costs[p] + costs[t];
        span = std::max(span, load);
      }
      if (span < best) { best = span; best_task = t; best_partner = p; }
    }
  }
  if (best_task < 0) return false;
  const int gt = a->task_to_gpu[best_task], gp = a->task_to_gpu[best_partner];
  a->gpus[gt].total_cost = a->gpus[gt].total_cost - costs[best_task] + costs[best_partner];
  a->gpus[gp].total_cost = a->gpus[gp].total_cost - costs[best_partner] + costs[best_task];
  a->task_to_gpu[best_task] = gp;
  a->task_to_gpu[best_partner] = gt;
  return true;
}

double ContiguousPartition::makespan() const {
  double m = 0.0;
  for (const RowShard& s : shards) m = std::max(m, s.total_cost);
  return m;
}

ContiguousPartition partition_rows_contiguous(const std::vector<RowTask>& rows, int num_gpus) {
  ContiguousPartition out;
  const int R = int(rows.size()), G = num_gpus;
  if (R <= 0 || G <= 0 || G > R) return out;

  std::vector<double> prefix(R + 1, 0.0);
  for (int i = 0; i < R; ++i) prefix[i + 1] = prefix[i] + rows[i].total_cost;

  // dp[g][i]: best makespan of rows [0, i) over g gpus; cut[g][i]: start row of
  // the last shard in that optimum.
  const size_t W = size_t(R) + 1;
  std::vector<double> dp(size_t(G + 1) * W, DBL_MAX);
  std::vector<int> cut(size_t(G + 1) * W, -1);
  dp[0] = 0.0;
  for (int g = 1; g <= G; ++g) {
    for (int i = 1; i <= R; ++i) {
      double& best = dp[size_t(g) * W + i];
      int& arg = cut[size_t(g) * W + i];
      for (int k = g - 1; k <= i - 1; ++k) {
        const double seg = prefix[i] - prefix[k];
        const double cand = std::max(dp[size_t(g - 1) * W + k], seg);
        if (cand < best) { best = cand; arg = k; }
      }
    }
  }

  out.shards.resize(G);
  out.row_to_gpu.assign(R, -1);
  int end = R;
  for (int g = G; g >= 1; --g) {
    const int begin = cut[size_t(g) * W + end];
    if (begin < 0) return ContiguousPartition{};
    RowShard& s = out.shards[g - 1];
    s.gpu = g - 1;
    s.row_begin = begin;
    s.row_end = end;
    s.total_cost = prefix[end] - prefix[begin];
    for (int r = begin; r < end; ++r) out.row_to_gpu[r] = g - 1;
    end = begin;
  }
  out.ok = true;
  return out;
}

}  // namespace mgfa::sched
