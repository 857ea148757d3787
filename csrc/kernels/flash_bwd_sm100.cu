// Attention backward on sm_100a tensor cores, head_dim 128, bf16 in, fp32 grads.
//
// Two kernels, no atomics (deterministic):
//   dK/dV: CTA = one 128-key tile of one kv head; loops over every visible
//          128-row query tile of every query head in its GQA group.
//            S^T  = K Q^T     (SS)        -> TMEM [0,128)
//            dP^T = V dO^T    (SS)        -> TMEM [128,256)
//            P^T  = exp2(S^T*scale_log2 - lse2)     (bf16, over S^T in TMEM)
//            dS^T = P^T * (dP^T - delta)           (bf16, over dP^T in TMEM)
//            dV  += P^T dO    (TS, dO MN-major)     -> TMEM [256,384)
//            dK  += dS^T Q    (TS, Q MN-major)      -> TMEM [384,512), * scale
//   dQ:    CTA = one 128-row query tile; loops over visible key tiles.
//            S  = Q K^T, dP = dO V^T (SS), dS = P * (dP - delta) written as bf16
//            over dP, dQ += dS K (TS, K MN-major), * scale at the end.
// MMA issue order lets the tensor core compute the next S while softmax
// threads work on the current tile (S is read into registers before the next
// S may overwrite it; P/dS buffers are consumed by MMAs issued earlier, and the
// tensor pipe runs a thread's MMAs in order).
// The reference prototype has no backward pass at all.
#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>

#include <cmath>

#include "flash_bwd_sm100.cuh"
#include "sm100_ptx.cuh"
#include "ring_push.cuh"

namespace mgfa {
namespace {

using namespace mgfa::dev;

constexpr int kTile = 128;
constexpr int kHalfBytes = kTile * 64 * 2;  // one 128 x 64 16-bit swizzled box
constexpr int kThreads = 192;  // 4 softmax warps, 1 TMA warp, 1 MMA warp

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int kD>
__device__ __forceinline__ void load_tile(void* dst, const CUtensorMap* m, uint64_t* bar, int h,
                                          int row, int b) {
  uint8_t* d = static_cast<uint8_t*>(dst);
#pragma unroll
  for (int hf = 0; hf < kD / 64; ++hf) tma_load_4d(d + hf * kHalfBytes, m, bar, hf * 64, h, row, b);
}

// K-major 128x128 operand (two 64-column swizzled halves), k-step kk of 16.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024);
}
// MN-major B operand: rows are the K dimension (128 B each), N halves 16 KB apart.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + kk * 2048, kHalfBytes, 1024);
}

template <int kN>
__device__ __forceinline__ void tmem_ld_cols(uint32_t addr, uint32_t (&r)[kN]) {
#pragma unroll
  for (int c = 0; c < kN; c += 32) tmem_ld32(addr + c, *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < kN; c += 32) regs_defined32(&r[c]);  // uses only after the wait
}

__device__ __forceinline__ void tmem_ld128(uint32_t addr, uint32_t (&r)[128]) {
  tmem_ld_cols<128>(addr, r);
}

template <int kD>
__device__ __forceinline__ void store_grad_row(float* dst, const uint32_t (&acc)[kD], float mul,
                                               bool accumulate) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int q4 = 0; q4 < kD / 4; ++q4) {
    float4 v = make_float4(__uint_as_float(acc[4 * q4]) * mul, __uint_as_float(acc[4 * q4 + 1]) * mul,
                           __uint_as_float(acc[4 * q4 + 2]) * mul,
                           __uint_as_float(acc[4 * q4 + 3]) * mul);
    if (accumulate) {
      const float4 o = d[q4];
      v.x += o.x;
      v.y += o.y;
      v.z += o.z;
      v.w += o.w;
    }
    d[q4] = v;
  }
}

// ====================================================================== dQ
template <int kD>
struct __align__(1024) DqSmem {
  uint16_t q[kTile * kD];
  uint16_t dout[kTile * kD];
  uint16_t k[2][kTile * kD];
  uint16_t v[2][kTile * kD];
  uint64_t qd_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full, s_free, dp_full, ds_full, dq_full, drain;
  uint32_t tmem_base;
  uint32_t abort_flag;
};

template <int kD, bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_dq_kernel(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_do,
                        const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const BwdParams p) {
  constexpr int kTileBytes = (kD / 64) * kHalfBytes;
  extern __shared__ uint8_t smem_raw[];
  DqSmem<kD>& s = *reinterpret_cast<DqSmem<kD>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t warp = warp_id(), lane = lane_id();
  // query tiles vary fastest: resident CTAs share one head's K/V in L2
  const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.hq / p.hkv);
  // key tiles [0, n_active) are visible to this query tile, [0, full_hi) unmasked
  const int q_tile_pos = p.causal ? __ldg(p.q_tile_pos + qt) : 0;
  const int n_active = p.causal ? visible_prefix(p.kv_tile_pos, p.n_kv_tiles, q_tile_pos + (kTile - 1))
                                : p.n_kv_tiles;
  if (n_active == 0 && p.accumulate && !p.consume.enabled) return;  // nothing to add

  AbortState ab{&s.abort_flag, p.status, p.wait_limit_ns};
  if (warp == 0) tmem_alloc<512>(&s.tmem_base);
  if (threadIdx.x == 0) {
    s.abort_flag = 0;
    mbar_init(&s.qd_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_free, 4);  // one arrive per softmax warp
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.ds_full, 4);
    mbar_init(&s.dq_full, 1);
    mbar_init(&s.drain, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t S_COL = 0, DP_COL = 128, DQ_COL = 256;

  if (warp == 4) {
    if (lane == 0 && n_active > 0) {
      mbar_arrive_expect_tx(&s.qd_full, 2 * kTileBytes);
      load_tile<kD>(s.q, &map_q, &s.qd_full, h, qt * kTile, b);
      load_tile<kD>(s.dout, &map_do, &s.qd_full, h, qt * kTile, b);
      int it = 0;
      int last_k[2] = {-1, -1}, last_v[2] = {-1, -1};
      for (int j = 0; j < n_active; ++j) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1, ab, 41)) break;
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        load_tile<kD>(s.k[st], &map_k, &s.k_full[st], hk, j * kTile, b);
        last_k[st] = int(ph);
        if (!mbar_wait(&s.v_empty[st], ph ^ 1, ab, 42)) break;
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        load_tile<kD>(s.v[st], &map_v, &s.v_full[st], hk, j * kTile, b);
        last_v[st] = int(ph);
        ++it;
      }
      volatile uint32_t never = 0;
      AbortState dab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.qd_full, 0, dab, 0);
      for (int st = 0; st < 2; ++st) {
        if (last_k[st] >= 0) mbar_wait(&s.k_full[st], uint32_t(last_k[st]), dab, 0);
        if (last_v[st] >= 0) mbar_wait(&s.v_full[st], uint32_t(last_v[st]), dab, 0);
      }
    }
  } else if (warp == 5) {
    if (lane == 0 && n_active > 0) {
      const uint32_t idesc_ss = make_idesc_16(128, 128, 0, 0, kF16);
      const uint32_t idesc_ts = make_idesc_16(128, kD, 0, 1, kF16);
      const uint32_t qb = smem_u32(s.q), db = smem_u32(s.dout);
      auto gemm_s = [&](int st) {
        const uint32_t kb = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + S_COL, kmajor_desc(qb, kk), kmajor_desc(kb, kk), idesc_ss, kk > 0);
      };
      auto gemm_dp = [&](int st) {
        const uint32_t vb = smem_u32(s.v[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + DP_COL, kmajor_desc(db, kk), kmajor_desc(vb, kk), idesc_ss, kk > 0);
      };
      bool ok = mbar_wait(&s.qd_full, 0, ab, 50) && mbar_wait(&s.k_full[0], 0, ab, 51);
      if (ok) {
        tc_fence_after();
        gemm_s(0);
        mma_commit(&s.s_full);
        ok = mbar_wait(&s.v_full[0], 0, ab, 52);
        if (ok) {
          tc_fence_after();
          gemm_dp(0);
          mma_commit(&s.dp_full);
        }
      }
      for (int it = 0; ok && it < n_active; ++it) {
        const int st = it & 1, st1 = (it + 1) & 1;
        const uint32_t ph1 = ((it + 1) >> 1) & 1;
        const bool more = it + 1 < n_active;
        if (more) {
          if (!(ok = mbar_wait(&s.k_full[st1], ph1, ab, 53))) break;
          if (!(ok = mbar_wait(&s.s_free, it & 1, ab, 54))) break;
          tc_fence_after();
          gemm_s(st1);
          mma_commit(&s.s_full);
        }
        if (!(ok = mbar_wait(&s.ds_full, it & 1, ab, 55))) break;
        tc_fence_after();
        const uint32_t kb = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(tmem + DQ_COL, tmem + DP_COL + kk * 8, mnmajor_desc(kb, kk), idesc_ts,
                 (it > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&s.k_empty[st]);
        mma_commit(&s.v_empty[st]);
        if (more) {
          if (!(ok = mbar_wait(&s.v_full[st1], ph1, ab, 56))) break;
          tc_fence_after();
          gemm_dp(st1);
          mma_commit(&s.dp_full);
        }
      }
      if (ok) mma_commit(&s.dq_full);
      mma_commit(&s.drain);
      volatile uint32_t never = 0;
      AbortState dab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.drain, 0, dab, 0);
    }
  } else if (warp < 4) {
    const int r = threadIdx.x;
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    const int row = qt * kTile + r;
    const bool row_valid = row < p.sq;
    const int64_t ml = (int64_t(b) * p.hq + h) * p.sq_pad + row;
    const float lse2 = p.lse2[ml];
    const float dlt = p.delta[ml];
    const int q_pos = q_tile_pos + r;
    int full_hi = p.n_kv_tiles - ((p.sk % kTile) != 0 ? 1 : 0);
    if (p.causal) {
      const int f = visible_prefix(p.kv_tile_pos, n_active, q_tile_pos - (kTile - 1));
      full_hi = f < full_hi ? f : full_hi;
    }
    bool ok = true;
    int it = 0;
    for (int j = 0; j < n_active; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full, it & 1, ab, 60));
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld128(tmem + lane_off + S_COL, sr);
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&s.s_free);
      float pr[128];
      if (j < full_hi) {  // warp-uniform fast path: no mask
        // one f32x2 FMA per pair of scores
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nl2 = f2_pack(-lse2, -lse2);
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, nl2),
                    x0, x1);
          pr[c] = ex2_approx(x0);
          pr[c + 1] = ex2_approx(x1);
        }
      } else {
        int n_vis = p.sk - j * kTile;
        if (p.causal) {
          const int lim = q_pos - __ldg(p.kv_tile_pos + j) + 1;
          n_vis = lim < n_vis ? lim : n_vis;
        }
        if (!row_valid) n_vis = 0;
#pragma unroll
        for (int c = 0; c < 128; ++c)
          pr[c] = (c < n_vis) ? ex2_approx(fmaf(__uint_as_float(sr[c]), p.scale_log2, -lse2)) : 0.f;
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&s.dp_full, it & 1, ab, 61));
      if (!ok) break;
      tc_fence_after();
      uint32_t pk[4][16];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t dpr[32];
        tmem_ld32(tmem + lane_off + DP_COL + ch * 32, dpr);
        tmem_wait_ld();
        regs_defined32(dpr);
        const uint64_t dl2 = f2_pack(dlt, dlt);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          // dS = P (dP - delta), one f32x2 subtract and multiply per pair
          float d0, d1;
          f2_unpack(f2_mul(f2_pack(pr[ch * 32 + 2 * c], pr[ch * 32 + 2 * c + 1]),
                           f2_sub(f2_pack(__uint_as_float(dpr[2 * c]),
                                          __uint_as_float(dpr[2 * c + 1])), dl2)),
                    d0, d1);
          pk[ch][c] = pack16<kF16>(d0, d1);
        }
        // dS over the first 64 columns of the dP region (column ch*16.. holds
        // keys ch*32 .. ch*32+31); the chunk just read is never overwritten before
        // it is read because chunk ch's output lands in columns [16ch, 16ch+16).
        tmem_st16(tmem + lane_off + DP_COL + ch * 16, pk[ch]);
      }
      tmem_wait_st();
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) regs_live16(pk[ch]);
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&s.ds_full);
      ++it;
    }
    if (n_active > 0 && ok) ok = __all_sync(0xffffffffu, mbar_wait(&s.dq_full, 0, ab, 62));
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    uint32_t acc[kD];
    if (n_active > 0 && ok) {
      tmem_ld_cols<kD>(tmem + lane_off + DQ_COL, acc);
    } else {
#pragma unroll
      for (int c = 0; c < kD; ++c) acc[c] = 0u;
    }
    if (row_valid && ok)
      store_grad_row<kD>(p.dq + int64_t(b) * p.dq_batch_stride + int64_t(row) * p.dq_row_stride +
                             int64_t(h) * kD,
                         acc, p.scale, p.accumulate != 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc<512>(tmem);
  if (p.consume.enabled && p.consume.done_counter && threadIdx.x == 0) {
    // the dQ kernel is the last reader of this step's slot: the last CTA re-arms
    // it and hands it back to the left neighbour
    __threadfence();
    const uint32_t prev = atomicAdd(p.consume.done_counter, 1u);
    if (prev == p.consume.done_target) {
      *p.consume.done_counter = 0u;
      if (p.consume.reset_arrivals) *p.consume.arrivals = 0u;
      fence_sys();
      st_release_sys(p.consume.left_credit, p.consume.left_credit_value);
    }
  }
}

// ====================================================================== dK / dV
template <int kD>
struct __align__(1024) DkvSmem {
  uint16_t k[kTile * kD];
  uint16_t v[kTile * kD];
  uint16_t q[2][kTile * kD];
  uint16_t dout[2][kTile * kD];
  float lse2[2][kTile];
  float delta[2][kTile];
  uint64_t kv_full;
  uint64_t qd_full[2], qd_empty[2];
  uint64_t s_full, dp_full, p_full, ds_full, dkv_full, drain;
  uint64_t trace[8];
  uint32_t tmem_base;
  uint32_t abort_flag;
};

template <int kD, bool kF16>
__global__ void __launch_bounds__(kDkdvThreads, 1)
    flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap map_q,
                          const __grid_constant__ CUtensorMap map_do,
                          const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_v, const BwdParams p) {
  constexpr int kTileBytes = (kD / 64) * kHalfBytes;
  extern __shared__ uint8_t smem_raw[];
  DkvSmem<kD>& s = *reinterpret_cast<DkvSmem<kD>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t warp = warp_id(), lane = lane_id();
  // key tiles vary fastest: resident CTAs share the group's Q/dO stream in L2
  const int j = gridDim.x - 1 - blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.hq / p.hkv;
  // query tiles [q_lo, n_q_tiles) see this key tile (a suffix: positions increase)
  const int kv_tile_pos = p.causal ? __ldg(p.kv_tile_pos + j) : 0;
  const int q_lo = p.causal ? visible_prefix(p.q_tile_pos, p.n_q_tiles, kv_tile_pos - kTile) : 0;
  const int n_q_active = p.n_q_tiles - q_lo;
  const int n_iter = n_q_active * G;
  if (n_iter == 0 && p.accumulate && !p.ring.enabled && !p.push.enabled) return;

  AbortState ab{&s.abort_flag, p.status, p.wait_limit_ns};
  if (warp == 0) tmem_alloc<512>(&s.tmem_base);
  if (threadIdx.x == 0) {
    s.abort_flag = 0;
    mbar_init(&s.kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.qd_full[i], 1);
      mbar_init(&s.qd_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.p_full, 4);  // one arrive per softmax warp
    mbar_init(&s.ds_full, 4);
    mbar_init(&s.dkv_full, 1);
    mbar_init(&s.drain, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t ST_COL = 0, DPT_COL = 128, DV_COL = 256, DK_COL = 256 + kD;

  if (warp == 4) {
    if (lane == 0 && n_iter > 0) {
      bool ok = true;
      if (p.consume.enabled) {  // K/V (and accumulators) of this step arrived?
        ok = wait_flag_geq(p.consume.arrivals, p.consume.arrivals_target, p.wait_limit_ns,
                           p.status, 70, 0);
        if (ok && p.consume.tag && ld_acquire_sys(p.consume.tag) != p.consume.expected_tag) {
          record_error(p.status, kErrTagMismatch, 70, 0);
          ok = false;
        }
        if (!ok) s.abort_flag = 1;
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      const bool kv_issued = ok;
      if (ok) {
        mbar_arrive_expect_tx(&s.kv_full, 2 * kTileBytes);
        load_tile<kD>(s.k, &map_k, &s.kv_full, hk, j * kTile, b);
        load_tile<kD>(s.v, &map_v, &s.kv_full, hk, j * kTile, b);
      }
      int it = 0;
      int last[2] = {-1, -1};
      for (int g = 0; ok && g < G; ++g) {
        const int h = hk * G + g;
        const int64_t mlbase = (int64_t(b) * p.hq + h) * p.sq_pad;
        for (int qt = q_lo; qt < p.n_q_tiles; ++qt) {
          const int st = it & 1;
          const uint32_t ph = (it >> 1) & 1;
          if (!(ok = mbar_wait(&s.qd_empty[st], ph ^ 1, ab, 71))) break;
          mbar_arrive_expect_tx(&s.qd_full[st], 2 * kTileBytes + 2 * kTile * 4);
          load_tile<kD>(s.q[st], &map_q, &s.qd_full[st], h, qt * kTile, b);
          load_tile<kD>(s.dout[st], &map_do, &s.qd_full[st], h, qt * kTile, b);
          bulk_load(s.lse2[st], p.lse2 + mlbase + qt * kTile, kTile * 4, &s.qd_full[st]);
          bulk_load(s.delta[st], p.delta + mlbase + qt * kTile, kTile * 4, &s.qd_full[st]);
          last[st] = int(ph);
          ++it;
        }
      }
      volatile uint32_t never = 0;
      AbortState dab{&never, nullptr, p.wait_limit_ns};
      if (kv_issued) mbar_wait(&s.kv_full, 0, dab, 0);
      for (int st = 0; st < 2; ++st)
        if (last[st] >= 0) mbar_wait(&s.qd_full[st], uint32_t(last[st]), dab, 0);
    }
  } else if (warp == 5) {
    if (lane == 0 && n_iter > 0) {
      const uint32_t idesc_ss = make_idesc_16(128, 128, 0, 0, kF16);
      const uint32_t idesc_ts = make_idesc_16(128, kD, 0, 1, kF16);
      const uint32_t kb = smem_u32(s.k), vb = smem_u32(s.v);
      auto gemm_st = [&](int st) {
        const uint32_t qb = smem_u32(s.q[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + ST_COL, kmajor_desc(kb, kk), kmajor_desc(qb, kk), idesc_ss, kk > 0);
      };
      auto gemm_dpt = [&](int st) {
        const uint32_t db = smem_u32(s.dout[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + DPT_COL, kmajor_desc(vb, kk), kmajor_desc(db, kk), idesc_ss, kk > 0);
      };
      bool ok = mbar_wait(&s.kv_full, 0, ab, 80) && mbar_wait(&s.qd_full[0], 0, ab, 81);
      if (ok) {
        tc_fence_after();
        gemm_st(0);
        mma_commit(&s.s_full);
        gemm_dpt(0);
        mma_commit(&s.dp_full);
      }
      for (int it = 0; ok && it < n_iter; ++it) {
        const int st = it & 1, st1 = (it + 1) & 1;
        const uint32_t ph1 = ((it + 1) >> 1) & 1;
        const bool more = it + 1 < n_iter;
        if (!(ok = mbar_wait(&s.p_full, it & 1, ab, 82))) break;
        tc_fence_after();
        const uint32_t db = smem_u32(s.dout[st]), qb = smem_u32(s.q[st]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(tmem + DV_COL, tmem + ST_COL + kk * 8, mnmajor_desc(db, kk), idesc_ts,
                 (it > 0 || kk > 0) ? 1u : 0u);
        if (more) {
          if (!(ok = mbar_wait(&s.qd_full[st1], ph1, ab, 83))) break;
          tc_fence_after();
          gemm_st(st1);
          mma_commit(&s.s_full);
        }
        if (!(ok = mbar_wait(&s.ds_full, it & 1, ab, 84))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(tmem + DK_COL, tmem + DPT_COL + kk * 8, mnmajor_desc(qb, kk), idesc_ts,
                 (it > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&s.qd_empty[st]);
        if (more) {
          gemm_dpt(st1);
          mma_commit(&s.dp_full);
        }
      }
      if (ok) mma_commit(&s.dkv_full);
      mma_commit(&s.drain);
      volatile uint32_t never = 0;
      AbortState dab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.drain, 0, dab, 0);
    }
  } else if (warp >= 6) {
    if (p.push.enabled)
      ring_push_warp(p.push, p.consume, p.status, p.wait_limit_ns, &s.abort_flag, s.trace,
                     int(warp) - 6);
  } else if (warp < 4) {
    const int r = threadIdx.x;  // key row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    const int key = j * kTile + r;
    const bool key_valid = key < p.sk;
    const int k_pos = kv_tile_pos + r;
    // query tiles [q_lo, q_full) are partially visible; [q_full, n) fully
    // (tile starts at or after this key tile's last key)
    const int q_full = p.causal ? visible_prefix(p.q_tile_pos, p.n_q_tiles, kv_tile_pos + kTile - 2)
                                : 0;
    bool ok = true;
    int it = 0;
    for (int g = 0; ok && g < G; ++g) {
      for (int qt = q_lo; qt < p.n_q_tiles; ++qt) {
        const int st = it & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full, it & 1, ab, 90));
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld128(tmem + lane_off + ST_COL, sr);
        // visible query columns c: q_pos(c) >= k_pos and the query row exists
        const float* lse2 = s.lse2[st];
        float pr[128];
        // rows past sq have lse2 = +inf (P = 0); keys past sk never get stored
        if (qt >= q_full && key_valid) {  // fast path: every query sees this key
#pragma unroll
          for (int c = 0; c < 128; ++c)
            pr[c] = ex2_approx(fmaf(__uint_as_float(sr[c]), p.scale_log2, -lse2[c]));
        } else {
          int c_lo = 0;
          if (p.causal) {
            const int lo = k_pos - __ldg(p.q_tile_pos + qt);
            c_lo = lo > 0 ? lo : 0;
          }
          const int c_hi = key_valid ? p.sq - qt * kTile : 0;  // exclusive
#pragma unroll
          for (int c = 0; c < 128; ++c)
            pr[c] = (c >= c_lo && c < c_hi)
                        ? ex2_approx(fmaf(__uint_as_float(sr[c]), p.scale_log2, -lse2[c]))
                        : 0.f;
        }
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) pk[c] = pack16<kF16>(pr[2 * c], pr[2 * c + 1]);
        tmem_st32(tmem + lane_off + ST_COL, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        tmem_st32(tmem + lane_off + ST_COL + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
        tmem_wait_st();
        regs_live32(&pk[0]);
        regs_live32(&pk[32]);
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.p_full);
        ok = __all_sync(0xffffffffu, mbar_wait(&s.dp_full, it & 1, ab, 91));
        if (!ok) break;
        tc_fence_after();
        const float* dl = s.delta[st];
        uint32_t dk[4][16];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t dpr[32];
          tmem_ld32(tmem + lane_off + DPT_COL + ch * 32, dpr);
          tmem_wait_ld();
          regs_defined32(dpr);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            // dS^T = P^T (dP^T - delta), one f32x2 subtract and multiply per pair
            const int c0 = ch * 32 + 2 * c;
            float d0, d1;
            f2_unpack(f2_mul(f2_pack(pr[c0], pr[c0 + 1]),
                             f2_sub(f2_pack(__uint_as_float(dpr[2 * c]),
                                            __uint_as_float(dpr[2 * c + 1])),
                                    f2_pack(dl[c0], dl[c0 + 1]))),
                      d0, d1);
            dk[ch][c] = pack16<kF16>(d0, d1);
          }
          tmem_st16(tmem + lane_off + DPT_COL + ch * 16, dk[ch]);
        }
        tmem_wait_st();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) regs_live16(dk[ch]);
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.ds_full);
        ++it;
      }
    }
    if (n_iter > 0 && ok) ok = __all_sync(0xffffffffu, mbar_wait(&s.dkv_full, 0, ab, 92));
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    uint32_t acc[kD];
    const int64_t off = int64_t(b) * p.dkv_batch_stride + int64_t(key) * p.dkv_row_stride +
                        int64_t(hk) * kD;
    if (n_iter > 0 && ok) {
      tmem_ld_cols<kD>(tmem + lane_off + DV_COL, acc);
    } else {
#pragma unroll
      for (int c = 0; c < kD; ++c) acc[c] = 0u;
    }
    if (!p.ring.enabled) {
      if (key_valid && ok) store_grad_row<kD>(p.dv + off, acc, 1.f, p.accumulate != 0);
      if (n_iter > 0 && ok) tmem_ld_cols<kD>(tmem + lane_off + DK_COL, acc);
      if (key_valid && ok) store_grad_row<kD>(p.dk + off, acc, p.scale, p.accumulate != 0);
    } else {
      // ring: out = incoming accumulator + this rank's contribution, stored into
      // the right neighbour's buffer once it is free
      volatile uint32_t* abort_flag = &s.abort_flag;
      if (lane == 0 && ok) {
        // the incoming accumulators must have arrived (a CTA without work gets
        // here before its neighbour is done) and the destination must be free
        if (p.consume.enabled &&
            !wait_flag_geq(p.consume.arrivals, p.consume.arrivals_target, p.wait_limit_ns,
                           p.status, 94, 0))
          *abort_flag = 1;
        if (!*abort_flag && !wait_flag_geq(p.ring.acc_credit, p.ring.acc_credit_target,
                                           p.wait_limit_ns, p.status, 93, 0))
          *abort_flag = 1;
      }
      __syncwarp();
      ok = __all_sync(0xffffffffu, ok && *abort_flag == 0);
      auto add_store = [&](float* dst, const float* src, float mul) {
        if (!MGFA_IN_BOUNDS(!p.ring.acc_out_elems || off + kD <= p.ring.acc_out_elems, p.status,
                            95))
          return;
        float4* d = reinterpret_cast<float4*>(dst + off);
        const float4* a = src ? reinterpret_cast<const float4*>(src + off) : nullptr;
#pragma unroll
        for (int q4 = 0; q4 < kD / 4; ++q4) {
          float4 v = make_float4(__uint_as_float(acc[4 * q4]) * mul,
                                 __uint_as_float(acc[4 * q4 + 1]) * mul,
                                 __uint_as_float(acc[4 * q4 + 2]) * mul,
                                 __uint_as_float(acc[4 * q4 + 3]) * mul);
          if (a) {
            const float4 o = a[q4];
            v.x += o.x;
            v.y += o.y;
            v.z += o.z;
            v.w += o.w;
          }
          d[q4] = v;
        }
      };
      if (key_valid && ok) add_store(p.ring.acc_out_dv, p.ring.acc_in_dv, 1.f);
      if (n_iter > 0 && ok) tmem_ld_cols<kD>(tmem + lane_off + DK_COL, acc);
      if (key_valid && ok) add_store(p.ring.acc_out_dk, p.ring.acc_in_dk, p.scale);
      // all four epilogue warps stored their rows: signal the neighbour once
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 0 && ok) {
        fence_sys();
        red_release_sys_add(p.ring.acc_arrivals, 1u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc<512>(tmem);
}

// ====================================================================== preprocess
template <int kD, bool kF16>
__global__ void bwd_preprocess_kernel(const uint16_t* __restrict__ o,
                                      const uint16_t* __restrict__ dout, int64_t o_sb,
                                      int64_t o_ss, int64_t do_sb, int64_t do_ss,
                                      const float* __restrict__ lse, int S, int H, int s_pad,
                                      float* __restrict__ lse2, float* __restrict__ delta) {
  // one warp per (b, h, row); row in [0, s_pad); lane handles kD / 32 elements
  constexpr int kPer = kD / 32;
  const int64_t wid = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= int64_t(H) * s_pad) return;
  const int row = int(wid % s_pad);
  const int h = int(wid / s_pad);
  const int b = blockIdx.y;
  float acc = 0.f;
  float l2 = INFINITY;
  if (row < S) {
    const uint16_t* op = o + b * o_sb + int64_t(row) * o_ss + int64_t(h) * kD + lane * kPer;
    const uint16_t* dp = dout + b * do_sb + int64_t(row) * do_ss + int64_t(h) * kD + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; i += 2) {
      const float2 a = unpack16<kF16>(*reinterpret_cast<const uint32_t*>(op + i));
      const float2 c = unpack16<kF16>(*reinterpret_cast<const uint32_t*>(dp + i));
      acc += a.x * c.x + a.y * c.y;
    }
    const float lv = lse[(int64_t(b) * H + h) * S + row];
    l2 = (lv == -INFINITY) ? INFINITY : lv * 1.4426950408889634f;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int64_t idx = (int64_t(b) * H + h) * s_pad + row;
    delta[idx] = acc;
    lse2[idx] = l2;
  }
}

template <class Kernel>
void set_smem(Kernel k, int smem, int& done_dev) {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (done_dev != dev) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    done_dev = dev;
  }
}

template <int kD, bool kF16>
void launch_dq(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
               const CUtensorMap& mv, const BwdParams& p, cudaStream_t stream) {
  static int done_dev = -1;
  const int smem = int(sizeof(DqSmem<kD>) + 1024);
  set_smem(flash_bwd_dq_kernel<kD, kF16>, smem, done_dev);
  flash_bwd_dq_kernel<kD, kF16><<<dim3(p.n_q_tiles, p.hq, p.batch), kThreads, smem, stream>>>(
      mq, mdo, mk, mv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int kD, bool kF16>
void launch_dkdv(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
                 const CUtensorMap& mv, const BwdParams& p, cudaStream_t stream) {
  static int done_dev = -1;
  const int smem = int(sizeof(DkvSmem<kD>) + 1024);
  set_smem(flash_bwd_dkdv_kernel<kD, kF16>, smem, done_dev);
  flash_bwd_dkdv_kernel<kD, kF16><<<dim3(p.n_kv_tiles, p.hkv, p.batch), kDkdvThreads, smem,
                                    stream>>>(mq, mdo, mk, mv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int kD, bool kF16>
void launch_preprocess(const void* o, const void* dout, int64_t o_sb, int64_t o_ss, int64_t do_sb,
                       int64_t do_ss, const float* lse, int B, int S, int H, int s_pad,
                       float* lse2, float* delta, cudaStream_t stream) {
  const int64_t warps = int64_t(H) * s_pad;
  const int threads = 256;
  dim3 grid(unsigned((warps * 32 + threads - 1) / threads), B);
  bwd_preprocess_kernel<kD, kF16><<<grid, threads, 0, stream>>>(
      static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(dout), o_sb, o_ss, do_sb,
      do_ss, lse, S, H, s_pad, lse2, delta);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

#define MGFA_BWD_DISPATCH(fn, ...)                                          \
  do {                                                                      \
    MGFA_CHECK(p.head_dim == 64 || p.head_dim == 128, "head_dim must be 64 or 128"); \
    if (p.head_dim == 64) {                                                 \
      if (p.fp16) fn<64, true>(__VA_ARGS__); else fn<64, false>(__VA_ARGS__); \
    } else {                                                                \
      if (p.fp16) fn<128, true>(__VA_ARGS__); else fn<128, false>(__VA_ARGS__); \
    }                                                                       \
  } while (0)

void flash_bwd_dq_launch(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
                         const CUtensorMap& mv, BwdParams& p, cudaStream_t stream) {
  MGFA_BWD_DISPATCH(launch_dq, mq, mdo, mk, mv, p, stream);
}

void flash_bwd_dkdv_launch(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
                           const CUtensorMap& mv, BwdParams& p, cudaStream_t stream) {
  MGFA_BWD_DISPATCH(launch_dkdv, mq, mdo, mk, mv, p, stream);
}

void flash_bwd_preprocess_launch(const void* o, const void* dout, int64_t o_sb, int64_t o_ss,
                                 int64_t do_sb, int64_t do_ss, const float* lse, int B, int S,
                                 int H, int s_pad, float* lse2, float* delta,
                                 cudaStream_t stream, int head_dim, bool fp16) {
  struct {
    int head_dim, fp16;
  } p{head_dim, fp16 ? 1 : 0};
  MGFA_BWD_DISPATCH(launch_preprocess, o, dout, o_sb, o_ss, do_sb, do_ss, lse, B, S, H, s_pad,
                    lse2, delta, stream);
}

}  // namespace mgfa

// ---------------------------------------------------------------------- no-throw launchers
// Used by the allocation-free C entry point (attn_bwd_noalloc.cu); they report
// errors through the return value instead of exceptions. They run the bf16,
// head_dim 128 kernels.
namespace mgfa {

cudaError_t flash_bwd_preprocess_raw(const void* o, const void* dout, int64_t o_sb, int64_t o_ss,
                                     int64_t do_sb, int64_t do_ss, const float* lse, int B, int S,
                                     int H, int s_pad, float* lse2, float* delta,
                                     cudaStream_t stream) {
  const int64_t warps = int64_t(H) * s_pad;
  const int threads = 256;
  dim3 grid(unsigned((warps * 32 + threads - 1) / threads), B);
  bwd_preprocess_kernel<128, false><<<grid, threads, 0, stream>>>(
      static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(dout), o_sb, o_ss, do_sb,
      do_ss, lse, S, H, s_pad, lse2, delta);
  return cudaGetLastError();
}

cudaError_t flash_bwd_kernels_raw(const CUtensorMap& mq, const CUtensorMap& mdo,
                                  const CUtensorMap& mk, const CUtensorMap& mv,
                                  const BwdParams& p, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(flash_bwd_dkdv_kernel<128, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(sizeof(DkvSmem<128>) + 1024));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(flash_bwd_dq_kernel<128, false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(sizeof(DqSmem<128>) + 1024));
  if (e != cudaSuccess) return e;
  flash_bwd_dkdv_kernel<128, false><<<dim3(p.n_kv_tiles, p.hkv, p.batch), kDkdvThreads,
                                      sizeof(DkvSmem<128>) + 1024, stream>>>(mq, mdo, mk, mv, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  flash_bwd_dq_kernel<128, false><<<dim3(p.n_q_tiles, p.hq, p.batch), kThreads,
                                    sizeof(DqSmem<128>) + 1024, stream>>>(mq, mdo, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace mgfa
