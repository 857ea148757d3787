// Parameters of the sm_100a attention forward kernel (shared by the launcher,
// the ring engine and the kernel).
#pragma once

#include <cuda.h>
#include <cstdint>

namespace mgfa {

// Optional in-kernel ring transport for one ring step: while the CTAs compute
// on the current KV shard, two warps per CTA push a slice of that shard into
// the right neighbour's receive slot with 16-byte stores through the peer
// mapping, then bumps the neighbour's arrival counter (release, system scope).
struct RingPush {
  const uint8_t* src_k = nullptr;  // current shard (local memory)
  const uint8_t* src_v = nullptr;
  uint8_t* dst_k = nullptr;        // right neighbour's slot (peer memory)
  uint8_t* dst_v = nullptr;
  uint64_t bytes = 0;              // bytes of K (== bytes of V); multiple of 16
  uint32_t* peer_arrivals = nullptr;  // right neighbour's arrival counter for that slot
  const uint32_t* credit = nullptr;   // local: right neighbour's uses of that slot finished
  uint32_t credit_target = 0;         // wait until *credit >= credit_target before writing
  uint32_t n_chunks = 0;              // chunks the shard is cut into (same on every rank);
                                      // CTAs with linear index < n_chunks push one each,
                                      // signalled in kFwdPushParts parts
  int enabled = 0;
  int drop_signal = 0;                // fault injection for tests: chunk 0 is copied but
                                      // never signalled, so the receiver's wait must expire
  uint32_t* peer_tag = nullptr;       // right neighbour's tag word for that slot
  uint32_t tag = 0;                   // (owner + 1) | (call << 8): written before signalling
  const uint8_t* dst_k_end = nullptr;  // ends of the destination buffers; debug builds
  const uint8_t* dst_v_end = nullptr;  // skip (and report) a store past them
};

// Consumer side of one ring step.
struct RingConsume {
  uint32_t* arrivals = nullptr;        // local arrival counter of the slot being read
  uint32_t arrivals_target = 0;        // wait until *arrivals >= target before reading;
                                       // the last CTA resets it to 0
  uint32_t* done_counter = nullptr;    // local counter of CTAs finished with this step;
                                       // null: only wait, a separate kernel releases
  uint32_t done_target = 0;            // value the last CTA sees (grid size - 1); it
                                       // resets the counter to 0
  uint32_t* left_credit = nullptr;     // left neighbour's credit word for this slot
  uint32_t left_credit_value = 0;      // value the last CTA publishes
  const uint32_t* tag = nullptr;       // tag word of the slot being read
  uint32_t expected_tag = 0;           // must match once the shard has arrived
  int reset_arrivals = 1;              // the release re-arms `arrivals` to 0; with 0
                                       // the count keeps growing and targets are
                                       // cumulative (set by the host)
  int enabled = 0;
};

struct FwdParams {
  int batch = 1, hq = 1, hkv = 1;
  int head_dim = 128;      // 64 or 128
  int fp16 = 0;            // inputs/outputs fp16 instead of bf16
  int sq = 0;              // query rows per sequence in this call
  int sk = 0;              // key rows per sequence in the KV buffer
  int n_q_tiles = 0, n_kv_tiles = 0;
  float scale_log2 = 0.f;  // softmax scale * log2(e)
  int causal = 0;
  const int* q_tile_pos = nullptr;   // [n_q_tiles]  global start of each 128-row query tile
  const int* kv_tile_pos = nullptr;  // [n_kv_tiles] global start of each 128-row key tile
  // outputs; row strides in elements, [B, S, H, D] order
  void* o = nullptr;                 // bf16 final output (when `final_out`)
  float* o_state = nullptr;          // fp32 running output (normalised)
  float* lse = nullptr;              // [B, Hq, sq] natural-log LSE
  int64_t o_batch_stride = 0, o_row_stride = 0;
  int merge = 0;                     // combine with the state already in o_state / lse
  int final_out = 1;                 // 1: write bf16 `o`; 0: write fp32 `o_state`
  uint32_t* status = nullptr;        // error word (0 = ok)
  uint64_t wait_limit_ns = 2000000000ull;
  RingPush push;
  RingConsume consume;
  // Optional per-CTA timeline (%globaltimer ns), kTraceWords u64 per CTA at
  // trace[linear_cta * kTraceWords]: {sm << 32 | cta, start, kv_ready,
  // epilogue, push_start, push_end, end, visible key tiles}.
  uint64_t* trace = nullptr;
  // Launched with programmatic dependent launch: the kernel may start while the
  // previous step's grid is still running; it waits for that grid only before
  // its epilogue touches the running state (o_state / lse / o).
  int dependent_launch = 0;
  // Pipeline: 0 whole 128-key tiles, packed f32x2 softmax; 1 half tiles (the
  // next half's S computed while the softmax works on the current one); 2
  // whole tiles, scalar softmax; -1 the build's default (or MGFA_FWD_VARIANT).
  // The launcher replaces -1 with the value it used.
  int variant = -1;
};

constexpr int kTraceWords = 8;
constexpr int kFwdPushParts = 2;  // push warps per CTA (arrivals per chunk)

// Host helpers (flash_fwd_sm100.cu).
// Tensor map of a [B, S, H, 128] bf16 tensor with the given element strides.
CUtensorMap make_bshd_map(const void* base, int64_t B, int64_t S, int64_t H,
                          int64_t stride_b, int64_t stride_s, int64_t stride_h);
// Same for head_dim `D` (64 or 128) and fp16 / bf16 elements.
CUtensorMap make_bshd_map_dt(const void* base, int64_t B, int64_t S, int64_t H,
                             int64_t stride_b, int64_t stride_s, int64_t stride_h, int D,
                             bool fp16);
void flash_fwd_launch_maps(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                           FwdParams& p, cudaStream_t stream);
int flash_fwd_grid_ctas(int hq, int n_q_tiles, int batch);

}  // namespace mgfa
