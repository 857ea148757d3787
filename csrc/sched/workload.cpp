#include "workload.hpp"

#include <algorithm>

namespace mgfa::sched {

const char* mask_name(MaskKind m) { return m == MaskKind::Causal ? "causal" : "full"; }

bool parse_mask(const std::string& s, MaskKind* out) {
  if (s == "causal") { *out = MaskKind::Causal; return true; }
  if (s == "full") { *out = MaskKind::Full; return true; }
  return false;
}

int num_row_blocks(const WorkloadShape& s) { return (s.seq_q + s.block_q - 1) / s.block_q; }
int num_col_blocks(const WorkloadShape& s) { return (s.seq_k + s.block_k - 1) / s.block_k; }
int64_t total_blocks(const WorkloadShape& s) {
  return int64_t(num_row_blocks(s)) * int64_t(num_col_blocks(s));
}

// Sum over q in [a, b) of (q - kb + 1), for kb <= a <= b.
static int64_t ramp_sum(int64_t a, int64_t b, int64_t kb) {
  if (b <= a) return 0;
  const int64_t hi = b - kb, lo = a - kb;
  return hi * (hi + 1) / 2 - lo * (lo + 1) / 2;
}

int64_t count_active(MaskKind m, int64_t qb, int64_t qe, int64_t kb, int64_t ke) {
  if (qe <= qb || ke <= kb) return 0;
  if (m == MaskKind::Full) return (qe - qb) * (ke - kb);
  // Causal: query q sees keys kb..min(q, ke-1).
  //   q <  kb       -> 0 keys
  //   kb <= q < ke  -> q - kb + 1 keys
  //   q >= ke       -> ke - kb keys
  const int64_t a = std::max(qb, kb), b = std::min(qe, ke);
  int64_t n = ramp_sum(a, b, kb);
  const int64_t full_from = std::max(qb, ke);
  if (qe > full_from) n += (qe - full_from) * (ke - kb);
  return n;
}

int64_t count_active_bruteforce(MaskKind m, int64_t qb, int64_t qe, int64_t kb, int64_t ke) {
  int64_t n = 0;
  for (int64_t q = qb; q < qe; ++q)
    for (int64_t k = kb; k < ke; ++k) n += mask_value(m, q, k);
  return n;
}

double estimate_cost(const CostModel& model, int64_t active) {
  if (active == 0) return 0.0;
  return model.alpha + model.beta * double(active);
}

std::vector<BlockTask> build_block_tasks(const WorkloadShape& s, MaskKind m,
                                         const CostModel& model, size_t max_tasks) {
  std::vector<BlockTask> tasks;
  const int rows = num_row_blocks(s), cols = num_col_blocks(s);
  for (int i = 0; i < rows; ++i) {
    const int qb = i * s.block_q, qe = std::min(qb + s.block_q, s.seq_q);
    for (int j = 0; j < cols; ++j) {
      const int kb = j * s.block_k, ke = std::min(kb + s.block_k, s.seq_k);
      const int64_t active = count_active(m, qb, qe, kb, ke);
      if (active == 0) continue;  // empty blocks carry no work
      if (tasks.size() >= max_tasks) return tasks;
      BlockTask t;
      t.row = i;
      t.col = j;
      t.q_begin = qb;
      t.q_end = qe;
      t.k_begin = kb;
      t.k_end = ke;
      t.active = active;
      t.total = int64_t(qe - qb) * int64_t(ke - kb);
      t.cost = estimate_cost(model, active);
      t.density = double(active) / double(t.total);
      tasks.push_back(t);
    }
  }
  return tasks;
}

std::vector<RowTask> build_row_tasks(const WorkloadShape& s, const std::vector<BlockTask>& tasks) {
  std::vector<RowTask> rows(num_row_blocks(s));
  for (size_t i = 0; i < rows.size(); ++i) rows[i].row = int(i);
  for (const BlockTask& t : tasks) {
    RowTask& r = rows[t.row];
    r.num_blocks += 1;
    r.comp_cost += t.cost;
    r.num_cols_needed = std::max(r.num_cols_needed, t.col + 1);
  }
  for (RowTask& r : rows) r.total_cost = r.comp_cost + r.comm_cost;
  return rows;
}

}  // namespace mgfa::sched
