// Native ring-attention forward engine (fused transport).
//
// One call runs the whole ring on the caller's stream: P launches of the
// sm_100a attention kernel, one per ring step. Step t computes the local
// queries against the KV shard of owner (rank - t) mod P (the reference's
// schedule, ring/attention/common/shard_utils.cuh:29-35) and, inside the same
// kernel, pushes that shard to the right neighbour's receive slot (t+1) % 3
// and merges its partial result into the running output. There is no host
// synchronisation between steps: ordering across ranks is carried entirely by
// the flag words of the symmetric buffer.
//
// Receive slots are triple-buffered: step t (t >= 1) reads slot t % 3 and
// pushes into the neighbour's slot (t + 1) % 3, whose previous use (step t - 2)
// finished long ago, so a push never waits on the neighbour's current step
// (the next step's CTAs start during this step's tail, see dependent launch).
// Flags (see comm/symmetric.hpp):
//   arrivals[s]  on the receiver, +1 per pushed chunk part; the kernels of a
//                step that reads slot s wait for all of them, the last CTA
//                rearms it
//   credit[s]    on the sender, the receiver's count of finished uses of its
//                slot s; a push into slot s waits until it equals the uses so
//                far (back-pressure)
//   done[s]      CTAs finished with slot s in this step (last CTA publishes)
// All ranks call forward() in the same order, so the per-slot use counts kept
// on the host agree everywhere.
#pragma once

#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdio>
#include <memory>

#include <nvtx3/nvToolsExt.h>

#include "../kernels/flash_fwd_sm100.cuh"
#include "ring_counters.hpp"
#include "symmetric.hpp"

namespace mgfa {

cudaError_t ring_push_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, int n_ctas, cudaStream_t stream);
cudaError_t ring_signal_launch(const RingPush& push, const RingConsume& consume,
                               cudaStream_t stream);
cudaError_t ring_wait_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, cudaStream_t stream);

class RingEngine {
 public:
  RingEngine(int rank, int world, int device, int64_t slot_bytes, int n_chunks)
      : buf_(size_t(2 * kSlots * slot_bytes), rank, world, device),
        slot_bytes_(size_t(slot_bytes)),
        n_chunks_(n_chunks) {
    MGFA_CHECK(slot_bytes > 0 && slot_bytes % 4096 == 0, "slot_bytes must be a multiple of 4096");
    // n_chunks: > 0 fixed, 0 two waves of CTAs, < 0 one chunk per CTA
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device));
  }

  std::string ipc_handle() const { return buf_.ipc_handle(); }

  void connect(const std::vector<std::string>& handles) { buf_.open_peers(handles); }

  int64_t slot_bytes() const { return int64_t(slot_bytes_); }
  std::vector<int64_t> uses() const {
    return {int64_t(ctr_.uses[0]), int64_t(ctr_.uses[1]), int64_t(ctr_.uses[2])};
  }

  // The flag values of `calls` consecutive transport calls on `rank` of a
  // `world`-rank ring, one row per step: {call, t, slot, next_slot,
  // credit_target, credit_value, tag}. Computed by the same RingCounters that
  // run() uses, without a GPU (checked against the protocol model).
  static std::vector<std::vector<int64_t>> plan(int world, int rank, int calls) {
    RingCounters c;
    std::vector<std::vector<int64_t>> rows;
    for (int k = 0; k < calls; ++k) {
      for (int t = 0; t < world; ++t) {
        const int owner = ((rank - t) % world + world) % world;
        const RingCounters::Step f = c.step(t, owner);
        rows.push_back({k, t, f.slot, f.next_slot, int64_t(f.credit_target),
                        int64_t(f.credit_value), int64_t(f.tag)});
        c.finish_step(t);
      }
      c.finish_call();
    }
    return rows;
  }

  // q [B,Sq,Hq,D]; k, v [B,L,Hkv,D] contiguous local shards, bf16 or fp16, D = 64 or
  // 128 (same L on every rank; owner o's first kv_lens[o] rows are valid).
  // kv_tile_pos [P, ceil(L/128)] int32: tile positions of each owner's shard as seen
  // from this rank's queries; q_tile_pos [ceil(Sq/128)] int32 (causal only).
  std::vector<torch::Tensor> forward(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                     double scale, bool causal,
                                     c10::optional<torch::Tensor> q_tile_pos,
                                     c10::optional<torch::Tensor> kv_tile_pos,
                                     std::vector<int64_t> kv_lens, torch::Tensor status,
                                     int64_t wait_limit_ns) {
    return run(q, k, v, scale, causal, q_tile_pos, kv_tile_pos, kv_lens, status, wait_limit_ns,
               /*transport=*/true);
  }

  // The same P launches with the transport switched off: every step computes on
  // the local shard with the step's masks and lengths. The gap to forward() is
  // the exposed communication time.
  std::vector<torch::Tensor> forward_compute_only(torch::Tensor q, torch::Tensor k,
                                                  torch::Tensor v, double scale, bool causal,
                                                  c10::optional<torch::Tensor> q_tile_pos,
                                                  c10::optional<torch::Tensor> kv_tile_pos,
                                                  std::vector<int64_t> kv_lens,
                                                  torch::Tensor status) {
    return run(q, k, v, scale, causal, q_tile_pos, kv_tile_pos, kv_lens, status,
               int64_t(2000000000), /*transport=*/false);
  }

 private:
  // n_chunks > 0: that many; 0: two waves of CTAs; < 0: one chunk per CTA.
  uint32_t push_chunks(int grid) const {
    if (n_chunks_ < 0) return uint32_t(grid);
    if (n_chunks_ > 0) return uint32_t(n_chunks_) < uint32_t(grid) ? uint32_t(n_chunks_) : uint32_t(grid);
    const uint32_t two_waves = 2u * uint32_t(num_sms_);
    return two_waves < uint32_t(grid) ? two_waves : uint32_t(grid);
  }

  std::vector<torch::Tensor> run(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                                 bool causal, c10::optional<torch::Tensor> q_tile_pos,
                                 c10::optional<torch::Tensor> kv_tile_pos,
                                 std::vector<int64_t> kv_lens, torch::Tensor status,
                                 int64_t wait_limit_ns, bool transport) {
    MGFA_CHECK(buf_.connected() || buf_.world() == 1, "RingEngine.connect() was not called");
    MGFA_CHECK(q.is_cuda() && (q.scalar_type() == at::kBFloat16 || q.scalar_type() == at::kHalf) &&
                    q.dim() == 4 && (q.size(3) == 128 || q.size(3) == 64) && q.is_contiguous(),
                "q must be a contiguous bf16/fp16 [B,S,H,64|128] CUDA tensor");
    MGFA_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type() &&
                    k.is_contiguous() && v.is_contiguous() && k.sizes() == v.sizes() &&
                    k.dim() == 4 && k.size(3) == q.size(3),
                "k and v must be contiguous tensors like q, [B,L,Hkv,D], of equal shape");
    const int P = buf_.world(), r = buf_.rank();
    const int right = (r + 1) % P, left = (r - 1 + P) % P;
    const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), L = k.size(1), Hkv = k.size(2);
    const int64_t D = q.size(3);
    const bool f16 = q.scalar_type() == at::kHalf;
    MGFA_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
    const size_t shard_bytes = size_t(B * L * Hkv * D * 2);
    MGFA_CHECK(P == 1 || shard_bytes <= slot_bytes_, "KV shard (", shard_bytes,
                " B) exceeds the engine's slot (", slot_bytes_, " B)");
    MGFA_CHECK(int64_t(kv_lens.size()) == P, "kv_lens needs one entry per rank");
    const int n_q_tiles = int((Sq + 127) / 128), n_kv_tiles = int((L + 127) / 128);
    if (causal) {
      MGFA_CHECK(q_tile_pos.has_value() && q_tile_pos->scalar_type() == at::kInt &&
                      q_tile_pos->numel() >= n_q_tiles,
                  "causal ring attention needs int32 q_tile_pos");
      MGFA_CHECK(kv_tile_pos.has_value() && kv_tile_pos->scalar_type() == at::kInt &&
                      kv_tile_pos->is_contiguous() && kv_tile_pos->dim() == 2 &&
                      kv_tile_pos->size(0) == P && kv_tile_pos->size(1) >= n_kv_tiles,
                  "causal ring attention needs int32 kv_tile_pos [P, n_kv_tiles]");
    }
    c10::cuda::CUDAGuard guard(q.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();

    auto o = torch::empty_like(q);
    auto lse = torch::empty({B, Hq, Sq}, q.options().dtype(at::kFloat));
    torch::Tensor o_state;
    if (P > 1) o_state = torch::empty(q.sizes(), q.options().dtype(at::kFloat));

    const CUtensorMap mq = make_bshd_map_dt(q.data_ptr(), B, Sq, Hq, q.stride(0), q.stride(1),
                                            q.stride(2), int(D), f16);
    const int64_t sb = L * Hkv * D, ss = Hkv * D, sh = D;
    auto slot_k = [&](int rank, int s) { return buf_.payload(rank) + size_t(s) * 2 * slot_bytes_; };
    auto slot_v = [&](int rank, int s) { return slot_k(rank, s) + slot_bytes_; };
    const int grid = flash_fwd_grid_ctas(int(Hq), n_q_tiles, int(B));
    if (trace_) {
      last_trace_ = torch::zeros({P, grid, kTraceWords}, q.options().dtype(at::kLong));
    }

    for (int t = 0; t < P; ++t) {
      const int owner = ((r - t) % P + P) % P;
      const RingCounters::Step f = ctr_.step(t, owner);
      const int s = f.slot;
      const bool own = t == 0 || !transport;
      const uint8_t* cur_k = own ? static_cast<const uint8_t*>(k.data_ptr()) : slot_k(r, s);
      const uint8_t* cur_v = own ? static_cast<const uint8_t*>(v.data_ptr()) : slot_v(r, s);
      const CUtensorMap mk = make_bshd_map_dt(cur_k, B, L, Hkv, sb, ss, sh, int(D), f16);
      const CUtensorMap mv = make_bshd_map_dt(cur_v, B, L, Hkv, sb, ss, sh, int(D), f16);

      FwdParams p;
      p.head_dim = int(D);
      p.fp16 = f16 ? 1 : 0;
      p.batch = int(B);
      p.hq = int(Hq);
      p.hkv = int(Hkv);
      p.sq = int(Sq);
      p.sk = int(kv_lens[owner]);
      p.n_q_tiles = n_q_tiles;
      p.n_kv_tiles = int((p.sk + 127) / 128);
      p.scale_log2 = float(scale * 1.4426950408889634);
      p.causal = causal ? 1 : 0;
      if (causal) {
        p.q_tile_pos = q_tile_pos->data_ptr<int>();
        p.kv_tile_pos = kv_tile_pos->data_ptr<int>() + int64_t(owner) * kv_tile_pos->size(1);
      }
      p.o = o.data_ptr();
      p.o_state = P > 1 ? o_state.data_ptr<float>() : nullptr;
      p.lse = lse.data_ptr<float>();
      p.o_batch_stride = q.stride(0);
      p.o_row_stride = q.stride(1);
      p.merge = t > 0 ? 1 : 0;
      p.final_out = t == P - 1 ? 1 : 0;
      p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
      p.wait_limit_ns = uint64_t(wait_limit_ns);
      // Steps after the first overlap the previous step's tail (dependent
      // launch); the first step of a call is fully ordered after everything
      // before it. Step t+1 releases its slot only after step t's grid is
      // complete (the epilogue's griddepcontrol.wait), but when a grid is
      // smaller than the SM count, steps t+1 and t+2 can be fully resident
      // while step t runs, so step t+3 could start and see step t's arrival
      // count on the slot they share before step t resets it (the owner tag
      // check would then fail the call). With P >= 5, where such a step t+3
      // exists, small grids therefore run without dependent launch.
      // (Cumulative arrival counts remove the hazard: a stale count never
      // reaches a later step's target.)
      const bool chain_hazard = !cumulative_ && P >= 5 && grid < num_sms_;
      p.dependent_launch = (t > 0 && pdl_ && !chain_hazard) ? 1 : 0;
      const bool unfused = transport && mode_ != kFusedPush;
      // chunks (= arrival signals) of the unfused transports
      const uint32_t x_chunks = mode_ == kCopyEngine ? 1u : uint32_t(2 * num_sms_);

      RingPush push_x;     // the standalone push kernel's (unfused transport)
      RingConsume wait_x;  // its wait for the slot it forwards
      if (transport && t < P - 1) {
        const int sn = f.next_slot;
        p.push.enabled = 1;
        p.push.src_k = cur_k;
        p.push.src_v = cur_v;
        p.push.dst_k = slot_k(right, sn);
        p.push.dst_v = slot_v(right, sn);
        p.push.dst_k_end = p.push.dst_k + slot_bytes_;
        p.push.dst_v_end = p.push.dst_v + slot_bytes_;
        p.push.bytes = shard_bytes;
        p.push.peer_arrivals = buf_.flag(right, comm::kArrivals0 + sn);
        p.push.credit = buf_.flag(r, comm::kCredit0 + sn);
        p.push.credit_target = f.credit_target;
        // The first chunks CTAs of the grid push (two waves by default, so the
        // shard reaches the neighbour early in the step). Every rank launches the
        // same grid (shards are padded to one length), so the receiver's arrival
        // target is the same number.
        p.push.n_chunks = push_chunks(grid);
        p.push.drop_signal = (drop_signal_step_ == t) ? 1 : 0;
        p.push.peer_tag = buf_.flag(right, comm::kTag0 + sn);
        p.push.tag = f.tag;
      }
      if (transport && t > 0) {
        p.consume.enabled = 1;
        p.consume.arrivals = buf_.flag(r, comm::kArrivals0 + s);
        const uint32_t per_use = unfused ? x_chunks : push_chunks(grid) * kFwdPushParts;
        if (cumulative_) {
          expected_[s] += per_use;
          p.consume.arrivals_target = expected_[s];
          p.consume.reset_arrivals = 0;
        } else {
          p.consume.arrivals_target = per_use;
        }
        p.consume.done_counter = buf_.flag(r, comm::kDone0 + s);
        p.consume.done_target = uint32_t(grid - 1);
        p.consume.left_credit = buf_.flag(left, comm::kCredit0 + s);
        p.consume.left_credit_value = f.credit_value;
        p.consume.tag = tag_check_ ? buf_.flag(r, comm::kTag0 + s) : nullptr;
        p.consume.expected_tag = f.tag;
      }
      if (unfused) {
        // Unfused transports: the same flags, but the shard moves on a second
        // stream -- in the standalone all-SM push kernel, or by the copy engine
        // (cudaMemcpyAsync into the peer slot between a one-thread wait kernel
        // and a one-thread signal kernel, no SMs for the data). The attention
        // kernel only waits for its slot, and a signal kernel releases the slot
        // once both the attention and the transfer are done with it. Step t+1's
        // attention is stream-ordered after step t's transfer, so a grid
        // spinning on its arrivals never holds SMs that a transfer it waits for
        // needs.
        p.dependent_launch = 0;
        push_x = p.push;
        push_x.n_chunks = x_chunks;
        push_x.peer_tag = nullptr;
        p.push = RingPush();
        if (t > 0) {
          p.consume.done_counter = nullptr;
          p.consume.tag = nullptr;
          wait_x = p.consume;
        }
      }
      if (trace_)
        p.trace = reinterpret_cast<uint64_t*>(last_trace_.data_ptr<int64_t>()) +
                  int64_t(t) * grid * kTraceWords;
      char label[64];
      std::snprintf(label, sizeof(label), "ring step %d (kv owner %d)", t, owner);
      nvtxRangePushA(label);
      cudaEvent_t pushed = nullptr;
      if (unfused && push_x.enabled) {
        if (!push_stream_) push_stream_ = c10::cuda::getStreamFromPool(false, buf_.device());
        cudaStream_t ps = push_stream_->stream();
        cudaEvent_t start;
        C10_CUDA_CHECK(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
        C10_CUDA_CHECK(cudaEventRecord(start, stream));
        C10_CUDA_CHECK(cudaStreamWaitEvent(ps, start, 0));
        C10_CUDA_CHECK(cudaEventDestroy(start));
        flash_fwd_launch_maps(mq, mk, mv, p, stream);
        if (mode_ == kCopyEngine) {
          // wait until the shard we forward has arrived and the right neighbour
          // has released the destination slot, copy, then signal one arrival
          C10_CUDA_CHECK(ring_wait_launch(push_x, wait_x, p.status, uint64_t(wait_limit_ns), ps));
          C10_CUDA_CHECK(cudaMemcpyAsync(push_x.dst_k, push_x.src_k, shard_bytes,
                                         cudaMemcpyDeviceToDevice, ps));
          C10_CUDA_CHECK(cudaMemcpyAsync(push_x.dst_v, push_x.src_v, shard_bytes,
                                         cudaMemcpyDeviceToDevice, ps));
          C10_CUDA_CHECK(ring_signal_launch(push_x, RingConsume(), ps));
        } else {
          C10_CUDA_CHECK(ring_push_launch(push_x, wait_x, p.status, uint64_t(wait_limit_ns),
                                          2 * num_sms_, ps));
        }
        C10_CUDA_CHECK(cudaEventCreateWithFlags(&pushed, cudaEventDisableTiming));
        C10_CUDA_CHECK(cudaEventRecord(pushed, ps));
        C10_CUDA_CHECK(cudaStreamWaitEvent(stream, pushed, 0));
        C10_CUDA_CHECK(cudaEventDestroy(pushed));
      } else {
        flash_fwd_launch_maps(mq, mk, mv, p, stream);
      }
      if (unfused && t > 0) {
        RingConsume rel;
        rel.enabled = 1;
        rel.arrivals = buf_.flag(r, comm::kArrivals0 + s);
        rel.left_credit = buf_.flag(left, comm::kCredit0 + s);
        rel.left_credit_value = f.credit_value;
        rel.reset_arrivals = cumulative_ ? 0 : 1;
        C10_CUDA_CHECK(ring_signal_launch(RingPush(), rel, stream));
      }
      nvtxRangePop();
      if (transport) ctr_.finish_step(t);
    }
    if (transport) ctr_.finish_call();
    return {o, lse};
  }

 public:
  // Transport of forward(): the attention kernel's push warps (fused, the
  // default), the standalone all-SM push kernel on a second stream, or the copy
  // engine on a second stream (the last two are ablations of the same flags).
  enum Mode : int { kFusedPush = 0, kPushKernel = 1, kCopyEngine = 2 };
  void set_transport_mode(int m) {
    MGFA_CHECK(m >= kFusedPush && m <= kCopyEngine, "transport mode must be 0, 1 or 2");
    mode_ = m;
  }
  int transport_mode() const { return mode_; }
  // Whether each consuming CTA verifies the slot's owner tag (one more
  // system-scope load before its first K load; on by default).
  void set_tag_check(bool on) { tag_check_ = on; }
  // Arrival counters that are never re-armed, with cumulative targets kept on
  // the host (off by default): dependent launch then stays on for every grid
  // size. Every rank must use the same setting; change it only right after
  // reset(). The 32-bit counts wrap after about 7 million uses of a slot.
  void set_cumulative_arrivals(bool on) { cumulative_ = on; }
  // false: the standalone push kernel (kept for callers of the two-way switch).
  void set_fused(bool on) { mode_ = on ? kFusedPush : kPushKernel; }
  bool fused() const { return mode_ == kFusedPush; }

 private:

 public:

  // Per-CTA kernel timelines of the following calls ([P, grid, 8] int64, see
  // FwdParams::trace), readable with last_trace().
  void set_trace(bool on) { trace_ = on; }
  // Programmatic dependent launch between ring steps (on by default).
  void set_dependent_launch(bool on) { pdl_ = on; }
  // Debug: NaN-fill this rank's receive slots (on the current stream), so that a
  // read racing ahead of its data shows up as NaNs in the next call's output.
  // Call only while the ring is quiescent on every rank (all ranks synchronised
  // and past a barrier; barrier again before the next call).
  void poison_slots() {
    c10::cuda::CUDAGuard guard(buf_.device());
    C10_CUDA_CHECK(cudaMemsetAsync(buf_.payload(buf_.rank()), 0xFF,
                                   size_t(2 * kSlots) * slot_bytes_,
                                   at::cuda::getCurrentCUDAStream()));
  }
  torch::Tensor last_trace() const { return last_trace_; }

  // Fault injection for tests (off by default): at ring step `step` of the next
  // forward calls, the push copies its data but skips one arrival signal.
  void set_drop_signal_step(int step) { drop_signal_step_ = step; }

  // Zero local flags and use counts (collective: every rank, then a barrier).
  void reset() {
    buf_.reset_flags(at::cuda::getCurrentCUDAStream());
    ctr_ = RingCounters();
    for (auto& e : expected_) e = 0;
  }

 private:
  comm::SymmetricBuffer buf_;
  size_t slot_bytes_;
  int n_chunks_;
  static constexpr int kSlots = RingCounters::kSlots;
  RingCounters ctr_;
  int drop_signal_step_ = -1;
  bool trace_ = false;
  bool pdl_ = true;
  int mode_ = kFusedPush;
  bool tag_check_ = true;
  bool cumulative_ = false;
  uint32_t expected_[kSlots] = {0, 0, 0};  // cumulative arrivals per slot (cumulative_)
  c10::optional<c10::cuda::CUDAStream> push_stream_;
  int num_sms_ = 148;
  torch::Tensor last_trace_;
};

}  // namespace mgfa
