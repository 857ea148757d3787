// Native ring-attention backward engine (fused transport).
//
// Step t (owner o = (rank - t) mod P) launches the dK/dV kernel and then the dQ
// kernel on the KV shard of o. The dK/dV kernel
//   * waits until slot t % 3 holds o's K, V and the dK/dV accumulators that the
//     ranks before it produced (t >= 1; the owner tag is checked),
//   * pushes K and V into the right neighbour's slot (t+1) % 3 with two warps
//     per CTA (the first two waves of CTAs),
//   * adds this rank's dK/dV contribution to the incoming accumulators and stores
//     the sums straight into the right neighbour's slot (t+1) % 3 -- or, at the
//     last step, into its home buffer, because the finished gradients of o then
//     belong to rank o = rank + 1 -- then signals once per CTA.
// The dQ kernel accumulates dQ locally; its last CTA re-arms slot t % 3 and
// hands it back to the left neighbour. After the last step the home buffer
// holds this rank's complete dK/dV (fp32), which are converted to bf16 before
// the home buffer is handed back. Slots are triple-buffered as in the forward.
#pragma once

#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <memory>

#include "../kernels/flash_bwd_sm100.cuh"
#include "ring_counters.hpp"
#include "symmetric.hpp"

namespace mgfa {

cudaError_t ring_wait_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, cudaStream_t stream);
cudaError_t ring_signal_launch(const RingPush& push, const RingConsume& consume,
                               cudaStream_t stream);

class RingBwdEngine {
 public:
  static constexpr int kSlots = 3;

  RingBwdEngine(int rank, int world, int device, int64_t kv_bytes, int n_chunks)
      : kv_bytes_(size_t((kv_bytes + 4095) / 4096 * 4096)),
        slot_bytes_(6 * kv_bytes_),
        buf_(size_t(kSlots) * 6 * kv_bytes_ + 4 * kv_bytes_, rank, world, device),
        n_chunks_(n_chunks) {
    MGFA_CHECK(kv_bytes > 0, "kv_bytes must be positive");
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device));
  }

  std::string ipc_handle() const { return buf_.ipc_handle(); }
  void connect(const std::vector<std::string>& handles) { buf_.open_peers(handles); }
  int64_t kv_bytes() const { return int64_t(kv_bytes_); }

  // The flag values of `calls` consecutive backward calls on `rank` of a
  // `world`-rank ring, one row per step: {call, t, slot, next_slot,
  // credit_target, credit_value, tag, home_credit_target}. Computed by the same
  // counters backward() uses, without a GPU (checked against the protocol model).
  static std::vector<std::vector<int64_t>> plan(int world, int rank, int calls) {
    RingCounters c;
    uint32_t home = 0;
    std::vector<std::vector<int64_t>> rows;
    for (int k = 0; k < calls; ++k) {
      for (int t = 0; t < world; ++t) {
        const int owner = ((rank - t) % world + world) % world;
        const RingCounters::Step f = c.step(t, owner);
        rows.push_back({k, t, f.slot, f.next_slot, int64_t(f.credit_target),
                        int64_t(f.credit_value), int64_t(f.tag | kBwdTag), int64_t(home)});
        c.finish_step(t);
      }
      home += 1;
      c.finish_call();
    }
    return rows;
  }

  void reset() {
    buf_.reset_flags(at::cuda::getCurrentCUDAStream());
    ctr_ = RingCounters();
    home_uses_ = 0;
  }

  // Returns (dq fp32 [B,L,Hq,128], dk fp32 [B,L,Hkv,128], dv fp32) for this rank's
  // shard; rows past the rank's own kv length are left unwritten.
  std::vector<torch::Tensor> backward(torch::Tensor dout, torch::Tensor q, torch::Tensor k,
                                      torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                                      double scale, bool causal,
                                      c10::optional<torch::Tensor> q_tile_pos,
                                      c10::optional<torch::Tensor> kv_tile_pos,
                                      std::vector<int64_t> kv_lens, torch::Tensor status,
                                      int64_t wait_limit_ns) {
    MGFA_CHECK(buf_.connected(), "RingBwdEngine.connect() was not called");
    const int64_t D = q.size(3);
    const bool f16 = q.scalar_type() == at::kHalf;
    for (auto* t : {&dout, &q, &k, &v, &out})
      MGFA_CHECK(t->is_cuda() && t->scalar_type() == q.scalar_type() &&
                      (q.scalar_type() == at::kBFloat16 || f16) && t->is_contiguous() &&
                      t->dim() == 4 && t->size(3) == D && (D == 64 || D == 128),
                  "dout/q/k/v/out must be contiguous bf16/fp16 [B,S,H,64|128] of one dtype");
    const int P = buf_.world(), r = buf_.rank();
    const int right = (r + 1) % P, left = (r - 1 + P) % P;
    const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), L = k.size(1), Hkv = k.size(2);
    const size_t kvb = size_t(B * L * Hkv * D * 2);
    MGFA_CHECK(kvb <= kv_bytes_, "KV shard exceeds the engine's buffers");
    MGFA_CHECK(int64_t(kv_lens.size()) == P, "kv_lens needs one entry per rank");
    const int n_q_tiles = int((Sq + 127) / 128), n_kv_tiles = int((L + 127) / 128);
    if (causal)
      MGFA_CHECK(q_tile_pos.has_value() && kv_tile_pos.has_value() &&
                      kv_tile_pos->size(0) == P && kv_tile_pos->size(1) >= n_kv_tiles,
                  "causal needs q_tile_pos and kv_tile_pos [P, n_kv_tiles]");
    c10::cuda::CUDAGuard guard(q.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();

    const int sq_pad = n_q_tiles * 128;
    auto f32 = q.options().dtype(at::kFloat);
    auto lse2 = torch::empty({B, Hq, sq_pad}, f32);
    auto delta = torch::empty({B, Hq, sq_pad}, f32);
    flash_bwd_preprocess_launch(out.data_ptr(), dout.data_ptr(), out.stride(0), out.stride(1),
                                dout.stride(0), dout.stride(1), lse.data_ptr<float>(), int(B),
                                int(Sq), int(Hq), sq_pad, lse2.data_ptr<float>(),
                                delta.data_ptr<float>(), stream, int(D), f16);
    auto dq = torch::empty(q.sizes(), f32);

    const int64_t sb = L * Hkv * D, ss = Hkv * D;
    const int64_t qsb = Sq * Hq * D, qss = Hq * D;
    const CUtensorMap mq = make_bshd_map_dt(q.data_ptr(), B, Sq, Hq, qsb, qss, D, int(D), f16);
    const CUtensorMap mdo = make_bshd_map_dt(dout.data_ptr(), B, Sq, Hq, qsb, qss, D, int(D), f16);
    auto slot = [&](int rank, int s) { return buf_.payload(rank) + size_t(s) * slot_bytes_; };
    auto home = [&](int rank) { return buf_.payload(rank) + size_t(kSlots) * slot_bytes_; };
    const int dkdv_grid = n_kv_tiles * int(Hkv) * int(B);
    const int dq_grid = n_q_tiles * int(Hq) * int(B);
    const uint32_t chunks = push_chunks(dkdv_grid);
    const uint32_t slot_target = chunks * kFwdPushParts + uint32_t(dkdv_grid);
    uint32_t* st = reinterpret_cast<uint32_t*>(status.data_ptr<int>());

    for (int t = 0; t < P; ++t) {
      const int owner = ((r - t) % P + P) % P;
      const RingCounters::Step f = ctr_.step(t, owner);
      const uint32_t step_tag = f.tag | kBwdTag;
      const int s = f.slot, sn = f.next_slot;
      const bool own = t == 0;
      const uint8_t* cur_k = own ? static_cast<const uint8_t*>(k.data_ptr()) : slot(r, s);
      const uint8_t* cur_v = own ? static_cast<const uint8_t*>(v.data_ptr()) : slot(r, s) + kv_bytes_;
      const CUtensorMap mk = make_bshd_map_dt(cur_k, B, L, Hkv, sb, ss, D, int(D), f16);
      const CUtensorMap mv = make_bshd_map_dt(cur_v, B, L, Hkv, sb, ss, D, int(D), f16);

      BwdParams p;
      p.head_dim = int(D);
      p.fp16 = f16 ? 1 : 0;
      p.batch = int(B);
      p.hq = int(Hq);
      p.hkv = int(Hkv);
      p.sq = int(Sq);
      p.sk = int(kv_lens[owner]);
      p.n_q_tiles = n_q_tiles;
      p.n_kv_tiles = int((p.sk + 127) / 128);
      p.sq_pad = sq_pad;
      p.scale = float(scale);
      p.scale_log2 = float(scale * 1.4426950408889634);
      p.causal = causal ? 1 : 0;
      if (causal) {
        p.q_tile_pos = q_tile_pos->data_ptr<int>();
        p.kv_tile_pos = kv_tile_pos->data_ptr<int>() + int64_t(owner) * kv_tile_pos->size(1);
      }
      p.lse2 = lse2.data_ptr<float>();
      p.delta = delta.data_ptr<float>();
      p.dq = dq.data_ptr<float>();
      p.dq_batch_stride = qsb;
      p.dq_row_stride = qss;
      p.dkv_batch_stride = sb;
      p.dkv_row_stride = ss;
      p.status = st;
      p.wait_limit_ns = uint64_t(wait_limit_ns);

      // ---- dK/dV: consume slot s, push K/V, move the accumulators
      BwdParams pk = p;
      if (t > 0) {
        pk.consume.enabled = 1;
        pk.consume.arrivals = buf_.flag(r, comm::kArrivals0 + s);
        pk.consume.arrivals_target = slot_target;
        pk.consume.tag = buf_.flag(r, comm::kTag0 + s);
        pk.consume.expected_tag = step_tag;
        pk.ring.acc_in_dk = reinterpret_cast<const float*>(slot(r, s) + 2 * kv_bytes_);
        pk.ring.acc_in_dv = reinterpret_cast<const float*>(slot(r, s) + 4 * kv_bytes_);
      }
      pk.ring.enabled = 1;
      // each accumulator region (slot or home) holds 2 * kv_bytes_ bytes of fp32
      pk.ring.acc_out_elems = int64_t(kv_bytes_ / 2);
      if (t < P - 1) {
        pk.push.enabled = 1;
        pk.push.src_k = cur_k;
        pk.push.src_v = cur_v;
        pk.push.dst_k = slot(right, sn);
        pk.push.dst_v = slot(right, sn) + kv_bytes_;
        pk.push.dst_k_end = pk.push.dst_v;
        pk.push.dst_v_end = slot(right, sn) + 2 * kv_bytes_;
        pk.push.bytes = kvb;
        pk.push.peer_arrivals = buf_.flag(right, comm::kArrivals0 + sn);
        pk.push.credit = buf_.flag(r, comm::kCredit0 + sn);
        pk.push.credit_target = f.credit_target;
        pk.push.n_chunks = chunks;
        pk.push.peer_tag = buf_.flag(right, comm::kTag0 + sn);
        pk.push.tag = step_tag;
        pk.ring.acc_out_dk = reinterpret_cast<float*>(slot(right, sn) + 2 * kv_bytes_);
        pk.ring.acc_out_dv = reinterpret_cast<float*>(slot(right, sn) + 4 * kv_bytes_);
        pk.ring.acc_arrivals = buf_.flag(right, comm::kArrivals0 + sn);
        pk.ring.acc_credit = buf_.flag(r, comm::kCredit0 + sn);
        pk.ring.acc_credit_target = f.credit_target;
      } else {  // the finished gradients of `owner` (= right) go home
        pk.ring.acc_out_dk = reinterpret_cast<float*>(home(right));
        pk.ring.acc_out_dv = reinterpret_cast<float*>(home(right) + 2 * kv_bytes_);
        pk.ring.acc_arrivals = buf_.flag(right, comm::kHomeArrivals);
        pk.ring.acc_credit = buf_.flag(r, comm::kHomeCredit);
        pk.ring.acc_credit_target = home_uses_;
      }
      flash_bwd_dkdv_launch(mq, mdo, mk, mv, pk, stream);

      // ---- dQ: accumulate locally; its last CTA releases slot s
      BwdParams pq = p;
      pq.accumulate = t > 0 ? 1 : 0;
      if (t > 0) {
        pq.consume.enabled = 1;
        pq.consume.arrivals = buf_.flag(r, comm::kArrivals0 + s);
        pq.consume.done_counter = buf_.flag(r, comm::kDone0 + s);
        pq.consume.done_target = uint32_t(dq_grid - 1);
        pq.consume.left_credit = buf_.flag(left, comm::kCredit0 + s);
        pq.consume.left_credit_value = f.credit_value;
      }
      flash_bwd_dq_launch(mq, mdo, mk, mv, pq, stream);
      ctr_.finish_step(t);
    }

    // ---- home: this rank's complete dK/dV arrived from the left neighbour
    RingPush none;
    RingConsume hc;
    hc.enabled = 1;
    hc.arrivals = buf_.flag(r, comm::kHomeArrivals);
    hc.arrivals_target = uint32_t(dkdv_grid);
    hc.left_credit = buf_.flag(left, comm::kHomeCredit);
    hc.left_credit_value = home_uses_ + 1;
    C10_CUDA_CHECK(ring_wait_launch(none, hc, st, uint64_t(wait_limit_ns), stream));
    auto opts = torch::TensorOptions().dtype(torch::kFloat).device(q.device());
    auto hk = torch::from_blob(home(r), {B, L, Hkv, D}, opts);
    auto hv = torch::from_blob(home(r) + 2 * kv_bytes_, {B, L, Hkv, D}, opts);
    auto dk = hk.clone();
    auto dv = hv.clone();
    C10_CUDA_CHECK(ring_signal_launch(none, hc, stream));  // hand the home buffer back
    home_uses_ += 1;
    ctr_.finish_call();
    return {dq, dk, dv};
  }

 private:
  uint32_t push_chunks(int grid) const {
    if (n_chunks_ < 0) return uint32_t(grid);
    if (n_chunks_ > 0) return uint32_t(n_chunks_) < uint32_t(grid) ? uint32_t(n_chunks_) : uint32_t(grid);
    const uint32_t two_waves = 2u * uint32_t(num_sms_);
    return two_waves < uint32_t(grid) ? two_waves : uint32_t(grid);
  }
  static constexpr uint32_t kBwdTag = 0x80000000u;  // backward tags differ from forward ones

  size_t kv_bytes_, slot_bytes_;
  comm::SymmetricBuffer buf_;
  int n_chunks_;
  int num_sms_ = 148;
  RingCounters ctr_;
  uint32_t home_uses_ = 0;
};

}  // namespace mgfa
