// Native ring-attention forward engine on the persistent kernel: the whole ring
// in ONE launch per call.
//
// Every rank keeps a receive slot for each ring step s = 1..P-1 (the shard of
// owner (rank - s) mod P, the reference's schedule from
// ring/attention/common/shard_utils.cuh:29-35), so no slot is reused within a
// call and no step waits for a neighbour to free one. The persistent kernel
// (kernels/attn_fwd_persistent.cu) computes every query tile against segment 0
// (the own shard) and then each received segment as soon as the kv-head chunk
// it needs has arrived, with the softmax state on chip across segments; its
// push warps forward every received chunk to the right neighbour's next slot.
//
// Flags (packed uint32 words in the symmetric buffer, see pflags):
//   arrivals[s][c]  parts of unit (segment s, kv-head chunk c) received from the
//                   left neighbour this call; the last CTA of the call waits
//                   for all of them and re-arms them to 0
//   tags[s][c]      (owner + 1) | call << 8 of the unit, checked by consumers
//   credit          calls the right neighbour has finished (it publishes call+1
//                   at the end of each call); a call's push waits until the
//                   right neighbour finished the previous one, i.e. its slots
//                   are free again
//   sched[2]        the kernel's work counter and finished-CTA count
// All ranks call forward() in the same order, so the call index agrees.
#pragma once

#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../kernels/attn_fwd_persistent.cuh"
#include "symmetric.hpp"

namespace mgfa {

CUtensorMap make_bshd_map_dt(const void* base, int64_t B, int64_t S, int64_t H, int64_t stride_b,
                             int64_t stride_s, int64_t stride_h, int D, bool fp16);

class RingEngineP {
 public:
  // shard_bytes: capacity of one K (or V) shard, B * L * Hkv * D * 2 bytes.
  RingEngineP(int rank, int world, int device, int64_t shard_bytes)
      : buf_(size_t(std::max(world - 1, 1)) * 2 * size_t(shard_bytes), rank, world, device,
             pflags::kBytes),
        shard_cap_(size_t(shard_bytes)) {
    MGFA_CHECK(world >= 1 && world <= kPMaxSeg, "ring size must be 1..16");
    MGFA_CHECK(shard_bytes > 0 && shard_bytes % 16 == 0, "shard_bytes must be a multiple of 16");
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device));
  }

  std::string ipc_handle() const { return buf_.ipc_handle(); }
  void connect(const std::vector<std::string>& handles) { buf_.open_peers(handles); }
  int64_t shard_bytes() const { return int64_t(shard_cap_); }
  int64_t calls() const { return int64_t(calls_); }
  int grid() const { return num_sms_; }

  // Flag values of `calls` consecutive calls on `rank` of a `world`-rank ring,
  // one row per call: {call, credit_target, credit_published, tag of segment 0,
  // ..., tag of segment world-1}. The same arithmetic forward() uses, without a
  // GPU (checked against the protocol model).
  static std::vector<std::vector<int64_t>> plan(int world, int rank, int calls) {
    std::vector<std::vector<int64_t>> rows;
    for (int k = 0; k < calls; ++k) {
      std::vector<int64_t> row = {k, k, k + 1};
      for (int s = 0; s < world; ++s) row.push_back(int64_t(seg_tag(world, rank, s, uint32_t(k))));
      rows.push_back(row);
    }
    return rows;
  }

  // q [B,Sq,Hq,D]; k, v [B,L,Hkv,D] contiguous local shards, bf16 or fp16, D = 64
  // or 128 (same L on every rank; owner o's first kv_lens[o] rows are valid).
  // kv_tile_pos [P, ceil(L/128)] int32 by owner; q_tile_pos [ceil(Sq/128)] int32
  // (causal only). Returns {o, lse}.
  std::vector<torch::Tensor> forward(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                     double scale, bool causal,
                                     c10::optional<torch::Tensor> q_tile_pos,
                                     c10::optional<torch::Tensor> kv_tile_pos,
                                     std::vector<int64_t> kv_lens, torch::Tensor status,
                                     int64_t wait_limit_ns) {
    return run(q, k, v, scale, causal, q_tile_pos, kv_tile_pos, kv_lens, status, wait_limit_ns,
               true);
  }

  // The same launch with the transport off: every segment reads the local shard
  // with its step's positions and length. The gap to forward() is the exposed
  // communication time.
  std::vector<torch::Tensor> forward_compute_only(torch::Tensor q, torch::Tensor k,
                                                  torch::Tensor v, double scale, bool causal,
                                                  c10::optional<torch::Tensor> q_tile_pos,
                                                  c10::optional<torch::Tensor> kv_tile_pos,
                                                  std::vector<int64_t> kv_lens,
                                                  torch::Tensor status) {
    return run(q, k, v, scale, causal, q_tile_pos, kv_tile_pos, kv_lens, status,
               int64_t(2000000000), false);
  }

  // Per-CTA timelines of the following calls ([grid, 8] int64 via last_trace()):
  // {sm << 32 | cta, start, end, items, ns waiting for arrivals, -, push start,
  // push end} (%globaltimer ns).
  void set_trace(bool on) { trace_ = on; }
  torch::Tensor last_trace() const { return last_trace_; }
  // Diagnostic knobs: the softmax variant word of the kernel (see
  // attn_fwd_persistent.cuh; -1 default) and whether push warps start only
  // after their CTA's compute.
  void set_tune(int tune) { tune_ = tune; }
  void set_push_after_compute(bool on) { push_after_ = on; }
  // Experiment knob: the last k CTAs only push, the others only compute (0: two
  // push warps in every CTA). Clamped to [0, grid / 2].
  void set_push_ctas(int k) { push_ctas_ = k < 0 ? 0 : k; }
  // Test knob: the next calls drop the signal of unit (segment 0, chunk 0),
  // part 0, so the right neighbour's wait for it must expire.
  void set_drop_signal(bool on) { drop_signal_ = on; }
  // Zero the local flags and the call count (collective: every rank, then a barrier).
  void reset() {
    buf_.reset_flags(at::cuda::getCurrentCUDAStream());
    calls_ = 0;
  }
  // Debug: NaN-fill this rank's receive slots (ring quiescent on every rank).
  void poison_slots() {
    c10::cuda::CUDAGuard guard(buf_.device());
    C10_CUDA_CHECK(cudaMemsetAsync(buf_.payload(buf_.rank()), 0xFF, buf_.payload_bytes(),
                                   at::cuda::getCurrentCUDAStream()));
  }

 private:
  static uint32_t seg_tag(int world, int rank, int s, uint32_t call) {
    const int owner = ((rank - s) % world + world) % world;
    return uint32_t(owner + 1) | (call << 8);
  }

  std::vector<torch::Tensor> run(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                                 bool causal, c10::optional<torch::Tensor> q_tile_pos,
                                 c10::optional<torch::Tensor> kv_tile_pos,
                                 std::vector<int64_t> kv_lens, torch::Tensor status,
                                 int64_t wait_limit_ns, bool transport) {
    const int P = buf_.world(), r = buf_.rank();
    MGFA_CHECK(buf_.connected() || P == 1, "RingEngineP.connect() was not called");
    MGFA_CHECK(q.is_cuda() && (q.scalar_type() == at::kBFloat16 || q.scalar_type() == at::kHalf) &&
                   q.dim() == 4 && (q.size(3) == 128 || q.size(3) == 64) && q.is_contiguous(),
               "q must be a contiguous bf16/fp16 [B,S,H,64|128] CUDA tensor");
    MGFA_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type() &&
                   k.is_contiguous() && v.is_contiguous() && k.sizes() == v.sizes() &&
                   k.dim() == 4 && k.size(3) == q.size(3) && k.size(0) == q.size(0),
               "k and v must be contiguous tensors like q, [B,L,Hkv,D], of equal shape");
    MGFA_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
               "status must be an int32 CUDA tensor");
    const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), L = k.size(1), Hkv = k.size(2);
    const int D = int(q.size(3));
    const bool f16 = q.scalar_type() == at::kHalf;
    MGFA_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
    MGFA_CHECK(B * Hkv <= kPMaxChunks, "batch * kv heads must be at most 2048");
    const uint64_t shard_bytes = uint64_t(B * L * Hkv * D * 2);
    MGFA_CHECK(P == 1 || shard_bytes <= shard_cap_, "KV shard (", shard_bytes,
               " B) exceeds the engine's capacity (", shard_cap_, " B)");
    MGFA_CHECK(int64_t(kv_lens.size()) == P, "kv_lens needs one entry per rank");
    const int n_q_tiles = int((Sq + 127) / 128), n_kv_tiles = int((L + 127) / 128);
    c10::cuda::CUDAGuard guard(q.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();

    PFwdParams p;
    p.batch = int(B);
    p.hq = int(Hq);
    p.hkv = int(Hkv);
    p.sq = int(Sq);
    p.n_q_tiles = n_q_tiles;
    p.n_items = int(B * Hq) * ((n_q_tiles + 1) / 2);
    p.n_seg = P;
    p.kv_rows = int(L);
    for (int s = 0; s < P; ++s) {
      const int owner = ((r - s) % P + P) % P;
      MGFA_CHECK(kv_lens[owner] >= 0 && kv_lens[owner] <= L, "kv_lens out of range");
      p.seg_len[s] = int(kv_lens[owner]);
    }
    p.scale_log2 = float(scale * 1.4426950408889634);
    p.causal = causal ? 1 : 0;
    if (causal) {
      MGFA_CHECK(q_tile_pos.has_value() && q_tile_pos->scalar_type() == at::kInt &&
                     q_tile_pos->is_contiguous() && q_tile_pos->numel() >= n_q_tiles,
                 "causal ring attention needs int32 q_tile_pos");
      MGFA_CHECK(kv_tile_pos.has_value() && kv_tile_pos->scalar_type() == at::kInt &&
                     kv_tile_pos->is_contiguous() && kv_tile_pos->dim() == 2 &&
                     kv_tile_pos->size(0) == P && kv_tile_pos->size(1) >= n_kv_tiles,
                 "causal ring attention needs int32 kv_tile_pos [P, n_kv_tiles]");
      p.q_tile_pos = q_tile_pos->data_ptr<int>();
      p.kv_tile_pos = by_segment(*kv_tile_pos).data_ptr<int>();
      p.kv_pos_stride = int(kv_tile_pos->size(1));
    }
    auto o = torch::empty_like(q);
    auto lse = torch::empty({B, Hq, Sq}, q.options().dtype(at::kFloat));
    p.o = o.data_ptr();
    p.lse = lse.data_ptr<float>();
    p.o_batch_stride = o.stride(0);
    p.o_row_stride = o.stride(1);
    p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
    p.wait_limit_ns = uint64_t(wait_limit_ns);
    p.sched = buf_.word(r, pflags::kSched);
    const int grid = num_sms_;
    if (trace_) {
      last_trace_ = torch::zeros({grid, kPTraceWords}, q.options().dtype(at::kLong));
      p.trace = reinterpret_cast<uint64_t*>(last_trace_.data_ptr<int64_t>());
    }

    const CUtensorMap mq = make_bshd_map_dt(q.data_ptr(), B, Sq, Hq, q.stride(0), q.stride(1),
                                            q.stride(2), D, f16);
    const int64_t sb = L * Hkv * D, ss = Hkv * D, sh = D;
    const CUtensorMap mk = make_bshd_map_dt(k.data_ptr(), B, L, Hkv, sb, ss, sh, D, f16);
    const CUtensorMap mv = make_bshd_map_dt(v.data_ptr(), B, L, Hkv, sb, ss, sh, D, f16);
    CUtensorMap mslots = mk;
    const bool ring = transport && P > 1;
    if (ring) {
      // slots 1..P-1 as one [2 (P-1) B, L, Hkv, D] tensor: segment s, K (kv = 0)
      // or V (kv = 1), batch b at outer index ((s - 1) * 2 + kv) * B + b
      mslots = make_bshd_map_dt(buf_.payload(r), 2 * (P - 1) * B, L, Hkv, sb, ss, sh, D, f16);
      const int right = (r + 1) % P, left = (r - 1 + P) % P;
      PRing& R = p.ring;
      R.enabled = 1;
      R.call = calls_;
      R.arrivals = buf_.word(r, pflags::kArrivals);
      R.tags = buf_.word(r, pflags::kTags);
      R.credit = buf_.word(r, pflags::kCredit);
      R.peer_arrivals = buf_.word(right, pflags::kArrivals);
      R.peer_tags = buf_.word(right, pflags::kTags);
      R.left_credit = buf_.word(left, pflags::kCredit);
      R.own_k = static_cast<const uint8_t*>(k.data_ptr());
      R.own_v = static_cast<const uint8_t*>(v.data_ptr());
      R.slots = buf_.payload(r);
      R.peer_slots = buf_.payload(right);
      R.peer_slots_end = R.peer_slots + size_t(P - 1) * 2 * shard_bytes;
      R.shard_bytes = shard_bytes;
      for (int s = 0; s < P; ++s) R.seg_tag[s] = seg_tag(P, r, s, calls_);
      R.drop_signal = drop_signal_ ? 1 : 0;
    }
    if (ring) {
      p.ring.push_after_compute = push_after_ ? 1 : 0;
      p.ring.push_ctas = push_ctas_ < grid / 2 ? push_ctas_ : grid / 2;
    }
    nvtxRangePushA(ring ? "ring attention (persistent)" : "ring attention compute only");
    attn_fwd_persistent_launch(mq, mk, mv, mslots, D, f16, p, grid, tune_, stream);
    nvtxRangePop();
    if (ring) calls_ += 1;
    return {o, lse};
  }

  // kv_tile_pos rows reordered from owners to segments (segment s = owner
  // (rank - s) mod P); cached for the caller's (cached) position table.
  const torch::Tensor& by_segment(const torch::Tensor& by_owner) {
    const int P = buf_.world(), r = buf_.rank();
    if (!pos_src_.defined() || !pos_src_.is_same(by_owner) ||
        pos_version_ != by_owner._version()) {
      std::vector<int64_t> idx(P);
      for (int s = 0; s < P; ++s) idx[s] = ((r - s) % P + P) % P;
      auto index = torch::tensor(idx, torch::dtype(torch::kLong)).to(by_owner.device());
      pos_seg_ = by_owner.index_select(0, index).contiguous();
      pos_src_ = by_owner;
      pos_version_ = by_owner._version();
    }
    return pos_seg_;
  }

  comm::SymmetricBuffer buf_;
  size_t shard_cap_;
  uint32_t calls_ = 0;
  int num_sms_ = 148;
  bool trace_ = false;
  bool drop_signal_ = false;
  int tune_ = -1;
  bool push_after_ = false;
  int push_ctas_ = 0;
  torch::Tensor last_trace_;
  torch::Tensor pos_src_, pos_seg_;
  uint32_t pos_version_ = 0;
};

}  // namespace mgfa
