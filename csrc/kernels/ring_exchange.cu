// Pure ring exchange (no attention math): one launch moves this rank's current
// slot into the right neighbour's other slot with 16-byte peer stores from
// every CTA, using the same arrival / credit protocol as the fused attention
// kernel (see flash_fwd_sm100.cuh), plus the two tiny flag kernels the
// copy-engine variant needs around cudaMemcpyAsync.
#include <cuda_runtime.h>

#include <cstdint>

#include "flash_fwd_sm100.cuh"
#include "sm100_ptx.cuh"

namespace mgfa {
namespace {

using namespace mgfa::dev;

__global__ void __launch_bounds__(512)
    ring_push_kernel(RingPush push, RingConsume consume, uint32_t* status, uint64_t limit_ns) {
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    if (consume.enabled &&
        !wait_flag_geq(consume.arrivals, consume.arrivals_target, limit_ns, status, 1, 0))
      abort_flag = 1;
    if (!abort_flag && push.enabled &&
        !wait_flag_geq(push.credit, push.credit_target, limit_ns, status, 2, 0))
      abort_flag = 1;
  }
  __syncthreads();
  if (!abort_flag && push.enabled) {
    const uint64_t total = 2 * push.bytes;
    const uint64_t chunk = ((total / push.n_chunks) + 15) & ~uint64_t(15);
    for (uint32_t c = blockIdx.x; c < push.n_chunks; c += gridDim.x) {
      const uint64_t b = uint64_t(c) * chunk;
      const uint64_t e = b + chunk < total ? b + chunk : total;
      const uint64_t stride = uint64_t(blockDim.x) * 16;
      for (uint64_t off = b + uint64_t(threadIdx.x) * 16; off < e; off += stride * 4) {
        uint4 r[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint64_t o = off + u * stride;
          if (o < e)
            r[u] = *reinterpret_cast<const uint4*>(o < push.bytes ? push.src_k + o
                                                                  : push.src_v + (o - push.bytes));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint64_t o = off + u * stride;
          if (o < e) {
            uint8_t* dst = o < push.bytes ? push.dst_k + o : push.dst_v + (o - push.bytes);
            [[maybe_unused]] const uint8_t* end = o < push.bytes ? push.dst_k_end : push.dst_v_end;
            if (MGFA_IN_BOUNDS(!end || dst + 16 <= end, status, 5))
              *reinterpret_cast<uint4*>(dst) = r[u];
          }
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        fence_sys();
        red_release_sys_add(push.peer_arrivals, 1u);
      }
    }
  }
  __syncthreads();
  if (consume.enabled && consume.done_counter && threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(consume.done_counter, 1u);
    if (prev == consume.done_target) {
      *consume.done_counter = 0u;
      if (consume.reset_arrivals) *consume.arrivals = 0u;
      fence_sys();
      st_release_sys(consume.left_credit, consume.left_credit_value);
    }
  }
}

// Copy-engine helpers: wait for (arrivals, credit) before the copy; signal after.
__global__ void ring_wait_kernel(RingPush push, RingConsume consume, uint32_t* status,
                                 uint64_t limit_ns) {
  if (consume.enabled)
    wait_flag_geq(consume.arrivals, consume.arrivals_target, limit_ns, status, 3, 0);
  if (push.enabled) wait_flag_geq(push.credit, push.credit_target, limit_ns, status, 4, 0);
}

__global__ void ring_signal_kernel(RingPush push, RingConsume consume) {
  if (push.enabled) {
    fence_sys();
    red_release_sys_add(push.peer_arrivals, push.n_chunks);
  }
  if (consume.enabled) {
    if (consume.reset_arrivals && consume.arrivals) *consume.arrivals = 0u;
    fence_sys();
    st_release_sys(consume.left_credit, consume.left_credit_value);
  }
}

}  // namespace

cudaError_t ring_push_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, int n_ctas, cudaStream_t stream) {
  ring_push_kernel<<<n_ctas, 512, 0, stream>>>(push, consume, status, limit_ns);
  return cudaGetLastError();
}

cudaError_t ring_wait_launch(const RingPush& push, const RingConsume& consume, uint32_t* status,
                             uint64_t limit_ns, cudaStream_t stream) {
  ring_wait_kernel<<<1, 1, 0, stream>>>(push, consume, status, limit_ns);
  return cudaGetLastError();
}

cudaError_t ring_signal_launch(const RingPush& push, const RingConsume& consume,
                               cudaStream_t stream) {
  ring_signal_kernel<<<1, 1, 0, stream>>>(push, consume);
  return cudaGetLastError();
}

}  // namespace mgfa
