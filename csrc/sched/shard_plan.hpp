// Token-shard ownership for ring attention.
//
// The reference gives rank r the contiguous ranges Q [r*n, (r+1)*n) and
// KV [r*n, (r+1)*n) and rotates KV to the right neighbour, so at ring step s
// rank r computes on the shard of owner (r - s) mod P and receives the shard of
// owner (r - s - 1) mod P (ring/attention/common/shard_utils.cuh:4-35).
//
// This plan generalises ownership to any layout in which every rank holds an
// ordered list of runs of consecutive global tokens:
//   contiguous  1 run per rank (the reference layout; uneven lengths allowed)
//   zigzag      2P chunks, rank r owns chunks r and 2P-1-r (causal balance)
//   striped     token t -> rank t mod P (a run of length 1 per token; the
//               kernels get a closed form instead of the run list)
//   scheduler   runs of `block` tokens taken from a row -> gpu map produced by
//               the workload schedulers (contiguous DP or row LPT)
// Q and KV use the same plan, so the KV shard of owner o holds exactly the
// tokens o owns as queries.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "workload.hpp"

namespace mgfa::sched {

enum class LayoutKind : int { Contiguous = 0, Zigzag = 1, Striped = 2, Scheduler = 3 };

const char* layout_name(LayoutKind k);
bool parse_layout(const std::string& s, LayoutKind* out);

struct TokenRun {
  int64_t gstart = 0;  // first global token position
  int64_t len = 0;
};

struct ShardPlan {
  LayoutKind kind = LayoutKind::Contiguous;
  int world = 1;
  int64_t seq = 0;
  std::vector<std::vector<TokenRun>> runs;  // per rank, local order (empty for striped)

  int64_t local_len(int rank) const;
  int64_t max_local_len() const;
  int64_t global_pos(int rank, int64_t local_index) const;
  std::vector<int64_t> positions(int rank) const;
  // Global start of each local tile of `tile` tokens, or -1 for a tile whose
  // tokens are not consecutive global positions. The kernels derive the causal
  // mask of a (query tile, key tile) pair from these two numbers.
  std::vector<int64_t> tile_starts(int rank, int tile) const;
  // Human-readable token set, "[a,b)" runs joined by '+', or "t%P==r" for striped.
  std::string describe(int rank) const;
  // Ring schedule (reference semantics).
  int compute_owner(int rank, int step) const { return ((rank - step) % world + world) % world; }
  int receive_owner(int rank, int step) const {
    return ((rank - step - 1) % world + world) % world;
  }
};

// Equal split when seq % world == 0; otherwise the first seq % world ranks get
// one extra token.
ShardPlan make_contiguous(int64_t seq, int world);
ShardPlan make_contiguous_lengths(const std::vector<int64_t>& lengths);
ShardPlan make_zigzag(int64_t seq, int world);  // seq % (2*world) == 0
ShardPlan make_striped(int64_t seq, int world);  // seq % world == 0
// Rank g owns the block rows with row_to_gpu[row] == g, in increasing order.
ShardPlan make_from_rows(int64_t seq, int block, const std::vector<int>& row_to_gpu, int world);
// Scheduler-driven plan: build the causal/full block workload over `seq`,
// partition it with the contiguous-row DP (policy "dp") or row LPT ("lpt") and
// convert the rows into runs.
ShardPlan make_scheduled(int64_t seq, int world, int block, MaskKind mask,
                         const std::string& policy, double beta = 1.0);

// Visible-score count of rank `q_rank`'s queries against owner `kv_rank`'s keys
// (the work of one ring step).
int64_t step_active(const ShardPlan& p, int q_rank, int kv_rank, MaskKind mask);

}  // namespace mgfa::sched
