#include "shard_plan.hpp"

#include <algorithm>
#include <stdexcept>

#include "scheduler.hpp"

namespace mgfa::sched {

const char* layout_name(LayoutKind k) {
  switch (k) {
    case LayoutKind::Contiguous: return "contiguous";
    case LayoutKind::Zigzag: return "zigzag";
    case LayoutKind::Striped: return "striped";
    case LayoutKind::Scheduler: return "scheduler";
  }
  return "?";
}

bool parse_layout(const std::string& s, LayoutKind* out) {
  if (s == "contiguous") *out = LayoutKind::Contiguous;
  else if (s == "zigzag") *out = LayoutKind::Zigzag;
  else if (s == "striped") *out = LayoutKind::Striped;
  else if (s == "scheduler") *out = LayoutKind::Scheduler;
  else return false;
  return true;
}

int64_t ShardPlan::local_len(int rank) const {
  if (kind == LayoutKind::Striped) return seq / world;
  int64_t n = 0;
  for (const TokenRun& r : runs.at(rank)) n += r.len;
  return n;
}

int64_t ShardPlan::max_local_len() const {
  int64_t m = 0;
  for (int r = 0; r < world; ++r) m = std::max(m, local_len(r));
  return m;
}

int64_t ShardPlan::global_pos(int rank, int64_t i) const {
  if (kind == LayoutKind::Striped) return i * world + rank;
  for (const TokenRun& r : runs.at(rank)) {
    if (i < r.len) return r.gstart + i;
    i -= r.len;
  }
  throw std::out_of_range("local index past the end of the shard");
}

std::vector<int64_t> ShardPlan::positions(int rank) const {
  std::vector<int64_t> out;
  out.reserve(size_t(local_len(rank)));
  if (kind == LayoutKind::Striped) {
    for (int64_t i = 0; i < seq / world; ++i) out.push_back(i * world + rank);
    return out;
  }
  for (const TokenRun& r : runs.at(rank))
    for (int64_t t = 0; t < r.len; ++t) out.push_back(r.gstart + t);
  return out;
}

std::vector<int64_t> ShardPlan::tile_starts(int rank, int tile) const {
  const int64_t n = local_len(rank);
  const int64_t ntiles = (n + tile - 1) / tile;
  std::vector<int64_t> out(size_t(ntiles), -1);
  if (kind == LayoutKind::Striped) return out;
  const std::vector<int64_t> pos = positions(rank);
  for (int64_t t = 0; t < ntiles; ++t) {
    const int64_t b = t * tile, e = std::min(n, b + tile);
    bool consecutive = true;
    for (int64_t i = b + 1; i < e && consecutive; ++i) consecutive = pos[i] == pos[i - 1] + 1;
    out[size_t(t)] = consecutive ? pos[size_t(b)] : -1;
  }
  return out;
}

std::string ShardPlan::describe(int rank) const {
  if (kind == LayoutKind::Striped)
    return "t%" + std::to_string(world) + "==" + std::to_string(rank);
  std::string s;
  for (const TokenRun& r : runs.at(rank)) {
    if (!s.empty()) s += "+";
    s += "[" + std::to_string(r.gstart) + "," + std::to_string(r.gstart + r.len) + ")";
  }
  return s.empty() ? "[0,0)" : s;
}

ShardPlan make_contiguous(int64_t seq, int world) {
  if (world <= 0 || seq < 0) throw std::invalid_argument("bad contiguous plan");
  std::vector<int64_t> lens(world, seq / world);
  for (int r = 0; r < int(seq % world); ++r) lens[r] += 1;
  return make_contiguous_lengths(lens);
}

ShardPlan make_contiguous_lengths(const std::vector<int64_t>& lengths) {
  ShardPlan p;
  p.kind = LayoutKind::Contiguous;
  p.world = int(lengths.size());
  p.runs.resize(lengths.size());
  int64_t at = 0;
  for (size_t r = 0; r < lengths.size(); ++r) {
    p.runs[r].push_back({at, lengths[r]});
    at += lengths[r];
  }
  p.seq = at;
  return p;
}

ShardPlan make_zigzag(int64_t seq, int world) {
  if (world <= 0 || seq % (2 * int64_t(world)) != 0)
    throw std::invalid_argument("zigzag needs seq divisible by 2*world");
  const int64_t c = seq / (2 * world);
  ShardPlan p;
  p.kind = LayoutKind::Zigzag;
  p.world = world;
  p.seq = seq;
  p.runs.resize(world);
  for (int r = 0; r < world; ++r) {
    p.runs[r].push_back({int64_t(r) * c, c});
    p.runs[r].push_back({int64_t(2 * world - 1 - r) * c, c});
  }
  return p;
}

ShardPlan make_striped(int64_t seq, int world) {
  if (world <= 0 || seq % world != 0) throw std::invalid_argument("striped needs seq % world == 0");
  ShardPlan p;
  p.kind = LayoutKind::Striped;
  p.world = world;
  p.seq = seq;
  p.runs.resize(world);
  return p;
}

ShardPlan make_from_rows(int64_t seq, int block, const std::vector<int>& row_to_gpu, int world) {
  ShardPlan p;
  p.kind = LayoutKind::Scheduler;
  p.world = world;
  p.seq = seq;
  p.runs.resize(world);
  for (size_t row = 0; row < row_to_gpu.size(); ++row) {
    const int g = row_to_gpu[row];
    if (g < 0 || g >= world) throw std::invalid_argument("row assigned to no gpu");
    const int64_t b = int64_t(row) * block, e = std::min<int64_t>(seq, b + block);
    std::vector<TokenRun>& rr = p.runs[g];
    if (!rr.empty() && rr.back().gstart + rr.back().len == b) rr.back().len += e - b;
    else rr.push_back({b, e - b});
  }
  return p;
}

ShardPlan make_scheduled(int64_t seq, int world, int block, MaskKind mask,
                         const std::string& policy, double beta) {
  const WorkloadShape shape{int(seq), int(seq), block, block};
  const std::vector<BlockTask> tasks = build_block_tasks(shape, mask, CostModel{0.0, beta});
  const std::vector<RowTask> rows = build_row_tasks(shape, tasks);
  if (policy == "dp") {
    const ContiguousPartition dp = partition_rows_contiguous(rows, world);
    if (!dp.ok) throw std::invalid_argument("contiguous DP needs at least one block row per gpu");
    return make_from_rows(seq, block, dp.row_to_gpu, world);
  }
  if (policy == "lpt") {
    const Assignment a = assign_row_lpt(rows, world, LptMode::Scan);
    return make_from_rows(seq, block, a.task_to_gpu, world);
  }
  throw std::invalid_argument("policy must be dp or lpt");
}

int64_t step_active(const ShardPlan& p, int q_rank, int kv_rank, MaskKind mask) {
  if (mask == MaskKind::Full) return p.local_len(q_rank) * p.local_len(kv_rank);
  if (p.kind == LayoutKind::Striped) {
    // local i <-> global i*P + r; key j visible iff j*P + o <= i*P + r.
    const int64_t n = p.seq / p.world;
    int64_t total = 0;
    for (int64_t i = 0; i < n; ++i) total += (kv_rank <= q_rank) ? (i + 1) : i;
    return total;
  }
  int64_t total = 0;
  for (const TokenRun& q : p.runs.at(q_rank))
    for (const TokenRun& k : p.runs.at(kv_rank))
      total += count_active(mask, q.gstart, q.gstart + q.len, k.gstart, k.gstart + k.len);
  return total;
}

}  // namespace mgfa::sched
