// In-kernel ring push used by the attention kernels: push warps copy this
// CTA's slice of the current KV shard into the right neighbour's receive slot
// (16-byte stores through the CUDA-IPC peer mapping) and signal each part with
// a system-scope release add on the neighbour's arrival counter.
#pragma once

#include "flash_fwd_sm100.cuh"
#include "sm100_ptx.cuh"

namespace mgfa {

constexpr int kPushWarps = kFwdPushParts;

using namespace mgfa::dev;

// Push warp `sub` of kPushWarps copies part `sub` of each of this CTA's chunks
// and signals it separately (the receiver waits for n_chunks * kPushWarps).
__device__ __forceinline__ void ring_push_warp(const RingPush& rp, const RingConsume& rc, uint32_t* status,
                               uint64_t limit_ns, volatile uint32_t* abort_flag,
                               uint64_t* trace_slots, int sub) {
  const uint32_t lane = lane_id();
  if (lane == 0) {
    // The shard we forward must have fully arrived here first...
    if (rc.enabled &&
        !wait_flag_geq(rc.arrivals, rc.arrivals_target, limit_ns, status, 11, 0))
      *abort_flag = 1;
    // ...and the right neighbour must be done with the slot we overwrite.
    if (!*abort_flag && !wait_flag_geq(rp.credit, rp.credit_target, limit_ns, status, 10, 0))
      *abort_flag = 1;
  }
  __syncwarp();
  if (*abort_flag) return;
  if (lane == 0 && sub == 0) trace_slots[4] = globaltimer();
  // The slot's owner tag: written (same value by every pushing CTA) before any
  // arrival signal, so a consumer that saw all arrivals also sees the tag.
  if (lane == 0 && rp.peer_tag) *reinterpret_cast<volatile uint32_t*>(rp.peer_tag) = rp.tag;
  const uint64_t total = 2 * rp.bytes;
  const uint64_t chunk = ((total / rp.n_chunks) + 15) & ~uint64_t(15);
  const uint32_t linear_cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const uint32_t n_ctas = gridDim.x * gridDim.y * gridDim.z;
  for (uint32_t c = linear_cta; c < rp.n_chunks; c += n_ctas) {
    const uint64_t cb = uint64_t(c) * chunk;
    const uint64_t ce = cb + chunk < total ? cb + chunk : total;
    const uint64_t part = (((ce > cb ? ce - cb : 0) / kPushWarps) + 15) & ~uint64_t(15);
    const uint64_t b0 = cb + uint64_t(sub) * part;
    const uint64_t b = b0 < ce ? b0 : ce;
    const uint64_t e = b + part < ce ? b + part : ce;
    // Copy [b, e) of the virtual concatenation K | V, 16 bytes per lane, 8 in flight.
    for (uint64_t off = b + uint64_t(lane) * 16; off < e; off += 32 * 16 * 8) {
      uint4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint64_t o = off + uint64_t(u) * 32 * 16;
        if (o < e) {
          const uint8_t* src = o < rp.bytes ? rp.src_k + o : rp.src_v + (o - rp.bytes);
          // plain (coherent) load: the slot was written by a peer in this epoch
          r[u] = *reinterpret_cast<const uint4*>(src);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint64_t o = off + uint64_t(u) * 32 * 16;
        if (o < e) {
          uint8_t* dst = o < rp.bytes ? rp.dst_k + o : rp.dst_v + (o - rp.bytes);
          [[maybe_unused]] const uint8_t* end = o < rp.bytes ? rp.dst_k_end : rp.dst_v_end;
          if (MGFA_IN_BOUNDS(!end || dst + 16 <= end, status, 12))
            *reinterpret_cast<uint4*>(dst) = r[u];
        }
      }
    }
    __syncwarp();
    if (lane == 0 && !(rp.drop_signal && c == 0)) {
      fence_sys();
      red_release_sys_add(rp.peer_arrivals, 1u);
    }
  }
  if (lane == 0 && sub == 0) trace_slots[5] = globaltimer();
}


}  // namespace mgfa
