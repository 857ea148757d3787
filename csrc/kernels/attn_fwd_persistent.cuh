// Parameters of the persistent sm_100a attention forward (attn_fwd_persistent.cu).
//
// One launch computes a query shard against a list of KV "segments": one for
// plain single-GPU attention, P for ring attention (segment s = the shard this
// rank holds at ring step s; the reference's schedule gives it owner
// (rank - s) mod P, ring/attention/common/shard_utils.cuh:29-35). The running
// softmax state of every (query tile, head) stays on chip across segments, so
// there is no per-step merge and the output is written once.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mgfa {

constexpr int kPMaxSeg = 16;         // KV segments per call (ring size <= 16)
constexpr int kPushUnitParts = 256;  // parts of one pushed unit (segment x kv-head chunk);
                                     // the receiver waits for all of them
constexpr int kPMaxChunks = 2048;    // batch * kv heads per call (flag array width)
constexpr int kPTraceWords = 8;

// Flag words of a persistent ring engine's symmetric buffer (uint32 indices).
namespace pflags {
constexpr int kCredit = 0;      // calls the right neighbour has finished reading its slots
constexpr int kSched = 32;      // [2] work counter, finished CTAs (this rank only)
constexpr int kArrivals = 2048; // [kPMaxSeg][kPMaxChunks] parts of each unit received
constexpr int kTags = kArrivals + kPMaxSeg * kPMaxChunks;  // [kPMaxSeg][kPMaxChunks]
constexpr int kWords = kTags + kPMaxSeg * kPMaxChunks;
constexpr size_t kBytes = size_t(kWords) * 4;
}  // namespace pflags

// In-kernel ring transport. Segment 0 is this rank's own shard (own_k / own_v);
// segment s >= 1 sits in local receive slot s. Every CTA's two push warps copy
// their parts of unit (s, chunk) -- the rows of one kv head of one batch entry
// of segment s, K and V -- into the right neighbour's slot s + 1 with 16-byte
// stores through the peer mapping, then release-add the neighbour's arrival
// counter of that unit. Units go in chunk-major order (all segments of kv head 0
// first), which is the order in which the heads are computed.
struct PRing {
  int enabled = 0;
  uint32_t call = 0;                 // index of this call since the last reset (same everywhere)
  uint32_t* arrivals = nullptr;      // local [kPMaxSeg][kPMaxChunks]
  const uint32_t* tags = nullptr;    // local [kPMaxSeg][kPMaxChunks]
  const uint32_t* credit = nullptr;  // local: right neighbour's finished calls
  uint32_t* peer_arrivals = nullptr; // right neighbour's arrival array
  uint32_t* peer_tags = nullptr;     // right neighbour's tag array
  uint32_t* left_credit = nullptr;   // left neighbour's credit word (we publish here)
  const uint8_t* own_k = nullptr;    // this rank's shard [B, L, Hkv, D]
  const uint8_t* own_v = nullptr;
  const uint8_t* slots = nullptr;    // local slots 1..P-1: [P-1][2 (K, V)][B, L, Hkv, D]
  uint8_t* peer_slots = nullptr;     // the right neighbour's slots (same layout)
  const uint8_t* peer_slots_end = nullptr;  // end of that region (debug bounds checks)
  uint64_t shard_bytes = 0;          // bytes of one K (or V) shard: B * L * Hkv * D * 2
  uint32_t seg_tag[kPMaxSeg] = {};   // tag of segment s's data: (owner + 1) | call << 8
  int drop_signal = 0;               // test knob: unit (segment 0, chunk 0) part 0 is
                                     // copied but never signalled
  int push_after_compute = 0;        // diagnostic knob: a CTA's push warps start only
                                     // once its softmax warps have finished every item
  int push_ctas = 0;                 // > 0: the last push_ctas CTAs of the grid only
                                     // push (all their warps) and compute nothing, and
                                     // the other CTAs only compute, so no CTA mixes the
                                     // two; 0: two push warps in every CTA
};

struct PFwdParams {
  int batch = 1, hq = 1, hkv = 1;
  int sq = 0;                        // query rows per sequence
  int n_q_tiles = 0;
  int n_items = 0;                   // batch * hq * ceil(n_q_tiles / 2)
  int n_seg = 1;
  int kv_rows = 0;                   // L: key rows per sequence in every KV buffer
  int seg_len[kPMaxSeg] = {};        // valid key rows of each segment (<= kv_rows)
  float scale_log2 = 0.f;            // softmax scale * log2(e)
  int causal = 0;
  const int* q_tile_pos = nullptr;   // [n_q_tiles]
  const int* kv_tile_pos = nullptr;  // [n_seg][kv_pos_stride]
  int kv_pos_stride = 0;
  void* o = nullptr;                 // [B, Sq, Hq, D] output (input dtype)
  float* lse = nullptr;              // [B, Hq, Sq] natural-log LSE
  int64_t o_batch_stride = 0, o_row_stride = 0;
  uint32_t* status = nullptr;
  uint64_t wait_limit_ns = 2000000000ull;
  uint32_t* sched = nullptr;         // [2] zero at launch; the last CTA re-arms them
  uint64_t* trace = nullptr;         // optional [grid][kPTraceWords]
  PRing ring;
};

// Host side (attn_fwd_persistent.cu). `tune` selects the softmax variant of
// the head_dim 128 bf16 kernel without the ring (every other kernel uses the
// default): bits 0-7 how many of every 8 exponential pairs run as a polynomial
// on the FMA pipe instead of MUFU.EX2 (0, 2 or 4), bits 8-9 the arithmetic
// (bit 8: packed f32x2) and the P hand-over (bit 9: two halves); bit 10 selects
// a variant that sums per-phase clock counts into `trace` ([grid][16] int64,
// layout in attn_fwd_persistent.cu), bit 11 computes the row max as a shallow
// tree, bit 12 computes the first half's exponentials speculatively against
// the running max, bit 13 hides the first P store's wait behind the next
// exponentials; negative means the default (0x100: packed f32x2 arithmetic,
// every exponential on MUFU, P handed over whole, which measured fastest at
// 32K-128K tokens under the power cap: the polynomial and the split hand-over
// add instructions that cost more clock than they save).
void attn_fwd_persistent_launch(const CUtensorMap& mq, const CUtensorMap& mk,
                                const CUtensorMap& mv, const CUtensorMap& mslots, int head_dim,
                                bool fp16, PFwdParams& p, int grid, int tune,
                                cudaStream_t stream);
int attn_fwd_persistent_smem_bytes(int head_dim);

}  // namespace mgfa
