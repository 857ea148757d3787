// Native pure ring exchange (the reference's ring/loop benchmarks, without MPI):
// a symmetric buffer with two slots per rank; step t sends slot t % 2 to the
// right neighbour's slot (t+1) % 2. Transports:
//   "p2p"  one all-SM push kernel per step (peer stores + arrival counters)
//   "ce"   copy engine: flag-wait kernel, cudaMemcpyAsync into the peer
//          mapping, flag-signal kernel
// The schedule and flags match the fused attention engine (ring_engine.cpp).
#pragma once

#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <memory>

#include "../kernels/flash_fwd_sm100.cuh"
#include "symmetric.hpp"

namespace mgfa {

cudaError_t ring_push_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, int n_ctas, cudaStream_t stream);
cudaError_t ring_wait_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, cudaStream_t stream);
cudaError_t ring_signal_launch(const RingPush& push, const RingConsume& consume,
                               cudaStream_t stream);

class RingExchange {
 public:
  RingExchange(int rank, int world, int device, int64_t slot_bytes, int n_ctas)
      : buf_(size_t(2 * slot_bytes), rank, world, device),
        slot_bytes_(size_t(slot_bytes)),
        n_ctas_(n_ctas) {
    MGFA_CHECK(slot_bytes > 0 && slot_bytes % 32 == 0, "slot_bytes must be a multiple of 32");
  }

  std::string ipc_handle() const { return buf_.ipc_handle(); }
  void connect(const std::vector<std::string>& handles) { buf_.open_peers(handles); }

  // uint8 view of this rank's slot s (for filling and checking).
  torch::Tensor slot(int s) {
    auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, buf_.device());
    return torch::from_blob(buf_.payload(buf_.rank()) + size_t(s & 1) * slot_bytes_,
                            {int64_t(slot_bytes_)}, opts);
  }

  // One ring step t on the current stream: send slot t%2 to the right
  // neighbour's slot (t+1)%2. `bytes` <= slot_bytes (multiple of 32).
  void step(int t, int64_t bytes, const std::string& transport, torch::Tensor status,
            int64_t wait_limit_ns) {
    MGFA_CHECK(buf_.connected(), "RingExchange.connect() was not called");
    MGFA_CHECK(bytes > 0 && size_t(bytes) <= slot_bytes_ && bytes % 32 == 0, "bad byte count");
    const int P = buf_.world(), r = buf_.rank();
    const int right = (r + 1) % P, left = (r - 1 + P) % P;
    const int s = t & 1, sn = (t + 1) & 1;
    c10::cuda::CUDAGuard guard(buf_.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    const uint32_t chunks = transport == "p2p" ? uint32_t(n_ctas_) : 1u;
    RingPush push;
    push.enabled = 1;
    const size_t half = size_t(bytes) / 2;  // "K" and "V" halves of the payload
    push.src_k = buf_.payload(r) + size_t(s) * slot_bytes_;
    push.src_v = push.src_k + half;
    push.dst_k = buf_.payload(right) + size_t(sn) * slot_bytes_;
    push.dst_v = push.dst_k + half;
    push.dst_k_end = push.dst_v;
    push.dst_v_end = push.dst_k + slot_bytes_;
    push.bytes = half;
    push.peer_arrivals = buf_.flag(right, comm::kArrivals0 + sn);
    push.credit = buf_.flag(r, comm::kCredit0 + sn);
    push.credit_target = uses_[sn];
    push.n_chunks = chunks;
    // Every step uses slot s and hands it back to the left neighbour once this
    // push has read it. At t > 0 the left neighbour filled it during step t-1,
    // so the push first waits for all its chunks; at t = 0 it holds this rank's
    // own data (no wait), which the left neighbour's step-1 push (P >= 3) must
    // not overwrite before this push is done -- hence the release at t = 0 too.
    RingConsume consume;
    consume.enabled = 1;
    consume.arrivals = buf_.flag(r, comm::kArrivals0 + s);
    consume.arrivals_target = t > 0 ? chunks : 0u;
    consume.done_counter = buf_.flag(r, comm::kDone0 + s);
    consume.done_target = uint32_t(n_ctas_ - 1);
    consume.left_credit = buf_.flag(left, comm::kCredit0 + s);
    consume.left_credit_value = uses_[s] + 1;
    uint32_t* st = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
    if (transport == "p2p") {
      C10_CUDA_CHECK(ring_push_launch(push, consume, st, uint64_t(wait_limit_ns), n_ctas_, stream));
    } else if (transport == "ce") {
      C10_CUDA_CHECK(ring_wait_launch(push, consume, st, uint64_t(wait_limit_ns), stream));
      C10_CUDA_CHECK(cudaMemcpyAsync(push.dst_k, push.src_k, size_t(bytes),
                                     cudaMemcpyDeviceToDevice, stream));
      C10_CUDA_CHECK(ring_signal_launch(push, consume, stream));
    } else {
      MGFA_CHECK(false, "transport must be p2p or ce");
    }
    uses_[s] += 1;
  }

  // Wait (on the current stream) until slot (t+1) % 2, which the left
  // neighbour fills during step t, has fully arrived. step(t) itself only waits
  // for the slot it forwards, so a caller that reads the received shard before
  // the next step must call this first. The counter stays armed for the
  // slot's next consumer (the next step or release()).
  void wait_received(int t, const std::string& transport, torch::Tensor status,
                     int64_t wait_limit_ns) {
    const int sn = (t + 1) & 1;
    c10::cuda::CUDAGuard guard(buf_.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    RingConsume arrived;
    arrived.enabled = 1;
    arrived.arrivals = buf_.flag(buf_.rank(), comm::kArrivals0 + sn);
    arrived.arrivals_target = transport == "p2p" ? uint32_t(n_ctas_) : 1u;
    uint32_t* st = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
    C10_CUDA_CHECK(ring_wait_launch(RingPush(), arrived, st, uint64_t(wait_limit_ns), stream));
  }

  // Finish with slot t % 2 after the last step: wait until it has fully
  // arrived, re-arm its counter and hand it back to the left neighbour (the data
  // stays readable until the next rotation overwrites it).
  void release(int t, const std::string& transport, torch::Tensor status,
               int64_t wait_limit_ns) {
    const int P = buf_.world(), r = buf_.rank();
    const int left = (r - 1 + P) % P, s = t & 1;
    c10::cuda::CUDAGuard guard(buf_.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    RingPush none;
    RingConsume consume;
    consume.enabled = 1;
    consume.arrivals = buf_.flag(r, comm::kArrivals0 + s);
    consume.arrivals_target = transport == "p2p" ? uint32_t(n_ctas_) : 1u;
    consume.left_credit = buf_.flag(left, comm::kCredit0 + s);
    consume.left_credit_value = uses_[s] + 1;
    uint32_t* st = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
    C10_CUDA_CHECK(ring_wait_launch(none, consume, st, uint64_t(wait_limit_ns), stream));
    C10_CUDA_CHECK(ring_signal_launch(none, consume, stream));
    uses_[s] += 1;
  }

  // A full rotation: P-1 steps, after which slot (P-1) % 2 holds the data of
  // owner (r+1) % P, then the release of that slot.
  void rotate(int64_t bytes, const std::string& transport, torch::Tensor status,
              int64_t wait_limit_ns) {
    const int P = buf_.world();
    for (int t = 0; t < P - 1; ++t) step(t, bytes, transport, status, wait_limit_ns);
    release(P - 1, transport, status, wait_limit_ns);
  }

  void reset() {
    buf_.reset_flags(at::cuda::getCurrentCUDAStream());
    uses_[0] = uses_[1] = 0;
  }

  int64_t slot_bytes() const { return int64_t(slot_bytes_); }

 private:
  comm::SymmetricBuffer buf_;
  size_t slot_bytes_;
  int n_ctas_;
  uint32_t uses_[2] = {0, 0};
};

}  // namespace mgfa
