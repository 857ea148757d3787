// Attention forward on sm_100a tensor cores (tcgen05 + TMEM + TMA), head_dim 128,
// bf16 in, fp32 accumulate, bf16 or fp32-state out, with
//   * causal masking from per-tile global token positions (contiguous, zigzag,
//     striped and scheduler-driven shards all reduce to this),
//   * an in-kernel LSE merge with the running output of earlier ring steps
//     (the reference merges with a separate kernel and normalises on the host:
//     ring/attention/bench/ring_attention_nccl_gpu_bench.cu:114-135, 398-407),
//   * an optional in-kernel ring push of the current KV shard to the right
//     neighbour's receive slot (peer stores + system-scope arrival counters).
//
// CTA = two 128-row query tiles of one (batch, head). Warp roles:
//   warps 0-3  softmax for query tile 0 (thread t owns row t / TMEM lane t)
//   warps 4-7  softmax for query tile 1
//   warp  8    TMA producer (Q once, then K and V tiles, 2-stage rings)
//   warp  9    MMA issuer (one thread): S = Q K^T (SS form), O += P V (TS form,
//              P read from TMEM where it overwrote S)
//   warps 10-11 ring push (only when a RingPush is enabled)
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512).
// Pipelines (template kVar):
//   kVar 0, whole tiles (the default): S_t(j) fills its 128 columns, P_t(j)
//     overwrites it, and the MMA order S0(j+1) after PV0(j), S1(j+1) after
//     PV1(j) lets one softmax warpgroup work while the tensor core runs the
//     other tile's GEMMs. The softmax uses packed f32x2 FMAs and adds (one
//     instruction per pair of scores).
//   kVar 2: kVar 0 with scalar fp32 softmax arithmetic.
//   kVar 1, half tiles: the 128 columns of tile t are two 64-key slots;
//     S_t(j, h) (N = 64) lands in slot h, P_t(j, h) overwrites it, and
//     S_t(j+1, h) is issued right after PV_t(j, h), so the next half is
//     computed while the softmax works on the current one. Measured slower
//     than kVar 0 on B200 (twice the S instructions at N = 64 and twice the
//     hand-overs outweigh the overlap), kept for comparison.
// O is rescaled only when the running max grows by more than 2^8 (the stale
// max keeps P <= 256, exact in fp32 sums and bf16 P).
#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>

#include <cmath>
#include <cstdlib>

#include "flash_fwd_sm100.cuh"
#include "sm100_ptx.cuh"
#include "softmax_exp.cuh"
#include "ring_push.cuh"
#include "tma_host.hpp"

namespace mgfa {
namespace {

using namespace mgfa::dev;

constexpr int kTile = 128;
constexpr int kHalfBytes = kTile * 64 * 2;   // one 128 x 64 16-bit swizzled box
constexpr int kWarps = 12;
constexpr int kThreads = kWarps * 32;
constexpr float kRescaleThreshold = 8.0f;    // log2 units
constexpr int kDefaultFwdVariant = 0;

// kD = head_dim (64 or 128) is kD / 64 swizzled 64-column boxes per 128-row tile.
template <int kD>
struct __align__(1024) FwdSmem {
  static constexpr int kHalves = kD / 64;
  uint16_t q[2][kHalves][kTile * 64];  // [query tile][d half], bf16 or fp16 bits
  uint16_t k[2][kHalves][kTile * 64];  // [stage][d half]
  uint16_t v[2][kHalves][kTile * 64];
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2];
  uint64_t sh_full[2][2], ph_full[2][2];  // half-tile pipeline: [query tile][slot]
  uint64_t o_done[2][2];  // half-tile pipeline: [query tile][key half], one phase per tile
  uint64_t o_full;
  uint64_t drain;
  uint64_t trace[kTraceWords];
  uint32_t tmem_base;
  uint32_t abort_flag;
};

__device__ __forceinline__ uint32_t sm_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// ------------------------------------------------------------------ kernel
// kD: head_dim (64 or 128); kF16: fp16 inputs/outputs (else bf16); kVar: the
// pipeline (0 whole tiles, 1 half tiles, 2 whole tiles with scalar fp32 softmax).
template <int kD, bool kF16, int kVar>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap map_q,
                     const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const FwdParams p) {
  constexpr int kHalves = kD / 64;
  constexpr int kTileBytes = kHalves * kHalfBytes;  // one 128 x kD tile
  constexpr int kKSteps = kD / 16;                  // MMA K steps of S = Q K^T
  constexpr int kOChunks = kD / 32;                 // 32-column TMEM chunks of O
  constexpr bool kHalfPipe = kVar == 1;
  constexpr bool kPackedExp = kVar != 2;
  extern __shared__ uint8_t smem_raw[];
  FwdSmem<kD>& s = *reinterpret_cast<FwdSmem<kD>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const uint32_t warp = warp_id(), lane = lane_id();
  // Query-tile pairs vary fastest so that the CTAs resident at one time work on
  // the same head and share its K/V stream in L2; heaviest pairs first (causal).
  const int pair = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y;                 // query head
  const int b = blockIdx.z;
  const int hk = h / (p.hq / p.hkv);
  const int qt0 = 2 * pair;

  // Key tiles [0, n_active) are visible to at least one of the CTA's query tiles;
  // tiles [0, full_hi[t]) are fully visible to query tile t (no mask needed).
  const bool has_q1 = qt0 + 1 < p.n_q_tiles;
  const int q_pos0 = p.causal ? __ldg(p.q_tile_pos + qt0) : 0;
  const int q_pos1 = (p.causal && has_q1) ? __ldg(p.q_tile_pos + qt0 + 1) : q_pos0;
  const int ragged = (p.sk % kTile) != 0 ? 1 : 0;
  int n_active = p.n_kv_tiles;
  if (p.causal)
    n_active = visible_prefix(p.kv_tile_pos, p.n_kv_tiles,
                              (q_pos0 > q_pos1 ? q_pos0 : q_pos1) + (kTile - 1));
  const bool has_prior = p.merge != 0;
  // No visible key tile: the running state is already correct unless this is
  // the final step, which still has to convert it to the 16-bit output.
  const bool skip_compute = n_active == 0;
  if (skip_compute && has_prior && !p.final_out && !p.push.enabled && !p.consume.enabled) return;

  // Let the next ring step's grid start filling SMs as this grid's CTAs retire.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  AbortState ab{&s.abort_flag, p.status, p.wait_limit_ns};
  if (warp == 0) tmem_alloc<512>(&s.tmem_base);
  if (threadIdx.x == 0) {
    s.abort_flag = 0;
    if (p.trace) {
      for (int i = 0; i < kTraceWords; ++i) s.trace[i] = 0;
      s.trace[1] = globaltimer();
    }
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], 4);  // one arrive per softmax warp
      for (int hh = 0; hh < 2; ++hh) {
        mbar_init(&s.sh_full[i][hh], 1);
        mbar_init(&s.ph_full[i][hh], 4);
      }
      mbar_init(&s.o_done[i][0], 1);
      mbar_init(&s.o_done[i][1], 1);
    }
    mbar_init(&s.o_full, 1);
    mbar_init(&s.drain, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 [256, 256+kD), O1 after it
  constexpr uint32_t kOCol = 256;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && !skip_compute) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      mbar_arrive_expect_tx(&s.q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int hf = 0; hf < kHalves; ++hf)
          tma_load_4d(s.q[t][hf], &map_q, &s.q_full, hf * 64, h, (qt0 + t) * kTile, b);
      bool ok = true;
      if (p.consume.enabled) {
        ok = wait_flag_geq(p.consume.arrivals, p.consume.arrivals_target, p.wait_limit_ns,
                           p.status, 8, 0);
        if (!ok) s.abort_flag = 1;
        // The shard must be the one this step expects (owner and call).
        if (ok && p.consume.tag && ld_acquire_sys(p.consume.tag) != p.consume.expected_tag) {
          record_error(p.status, kErrTagMismatch, 8, 0);
          s.abort_flag = 1;
          ok = false;
        }
        // Data written by peers' generic stores, read here by the async proxy.
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      if (p.trace) s.trace[2] = globaltimer();
      int it = 0;
      int last_k_phase[2] = {-1, -1}, last_v_phase[2] = {-1, -1};
      for (int j = 0; ok && j < n_active; ++j) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1, ab, 81)) break;
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        for (int hf = 0; hf < kHalves; ++hf)
          tma_load_4d(s.k[st][hf], &map_k, &s.k_full[st], hf * 64, hk, j * kTile, b);
        last_k_phase[st] = int(ph);
        if (!mbar_wait(&s.v_empty[st], ph ^ 1, ab, 82)) break;
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        for (int hf = 0; hf < kHalves; ++hf)
          tma_load_4d(s.v[st][hf], &map_v, &s.v_full[st], hf * 64, hk, j * kTile, b);
        last_v_phase[st] = int(ph);
        ++it;
      }
      // Drain: never leave the CTA with a TMA write outstanding.
      volatile uint32_t never = 0;
      AbortState drain_ab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.q_full, 0, drain_ab, 0);
      for (int st = 0; st < 2; ++st) {
        if (last_k_phase[st] >= 0) mbar_wait(&s.k_full[st], uint32_t(last_k_phase[st]), drain_ab, 0);
        if (last_v_phase[st] >= 0) mbar_wait(&s.v_full[st], uint32_t(last_v_phase[st]), drain_ab, 0);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && !skip_compute) {
      const uint32_t idesc_s = make_idesc_16(128, 128, 0, 0, kF16);
      const uint32_t idesc_o = make_idesc_16(128, kD, 0, 1, kF16);
      const uint32_t q_base[2] = {smem_u32(s.q[0][0]), smem_u32(s.q[1][0])};
      auto issue_s = [&](int t, int st) {
        const uint32_t kb = smem_u32(s.k[st][0]);
#pragma unroll
        for (int kk = 0; kk < kKSteps; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_ss(tmem + t * 128, make_sdesc_sw128(q_base[t] + off, 16, 1024),
                 make_sdesc_sw128(kb + off, 16, 1024), idesc_s, kk > 0);
        }
      };
      auto issue_o = [&](int t, int st, uint32_t acc) {
        const uint32_t vb = smem_u32(s.v[st][0]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 128 keys, 16 per step
          mma_ts(tmem + kOCol + t * kD, tmem + t * 128 + kk * 8,
                 make_sdesc_sw128(vb + kk * 2048, kHalfBytes, 1024), idesc_o,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      // half-tile pipeline: S_t(j, hh) = Q_t K(j)[64 hh, 64 hh + 64)^T into slot hh
      const uint32_t idesc_s64 = make_idesc_16(128, 64, 0, 0, kF16);
      auto issue_s_half = [&](int t, int st, int hh) {
        const uint32_t kb = smem_u32(s.k[st][0]) + uint32_t(hh) * 64 * 128;
#pragma unroll
        for (int kk = 0; kk < kKSteps; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_ss(tmem + t * 128 + hh * 64, make_sdesc_sw128(q_base[t] + off, 16, 1024),
                 make_sdesc_sw128(kb + off, 16, 1024), idesc_s64, kk > 0);
        }
      };
      // O_t += P_t(j, hh) V(j)[64 hh, 64 hh + 64)
      auto issue_o_half = [&](int t, int st, int hh, uint32_t acc) {
        const uint32_t vb = smem_u32(s.v[st][0]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tmem + kOCol + t * kD, tmem + t * 128 + hh * 64 + kk * 8,
                 make_sdesc_sw128(vb + (hh * 4 + kk) * 2048, kHalfBytes, 1024), idesc_o,
                 (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(&s.q_full, 0, ab, 90);
      if (ok) ok = mbar_wait(&s.k_full[0], 0, ab, 91);
      if (ok) {
        tc_fence_after();
        if constexpr (kHalfPipe) {
          for (int hh = 0; hh < 2; ++hh)
            for (int t = 0; t < 2; ++t) {
              issue_s_half(t, 0, hh);
              mma_commit(&s.sh_full[t][hh]);
            }
        } else {
          issue_s(0, 0);
          mma_commit(&s.s_full[0]);
          issue_s(1, 0);
          mma_commit(&s.s_full[1]);
        }
        mma_commit(&s.k_empty[0]);
      }
      // Half tiles: PV_0(j,0) S_0(j+1,0) PV_1(j,0) S_1(j+1,0) PV_0(j,1) S_0(j+1,1)
      // PV_1(j,1) S_1(j+1,1). S_t(j+1, hh) reuses slot hh right after the PV that
      // read P_t(j, hh) from it (the tensor core runs them in issue order).
      for (int it = 0; kHalfPipe && ok && it < n_active; ++it) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const int st1 = (it + 1) & 1;
        const uint32_t ph1 = ((it + 1) >> 1) & 1;
        const bool more = it + 1 < n_active;
        if (!(ok = mbar_wait(&s.v_full[st], ph, ab, 92))) break;
        bool k_next = false;
        for (int hh = 0; ok && hh < 2; ++hh) {
          for (int t = 0; t < 2; ++t) {
            if (!(ok = mbar_wait(&s.ph_full[t][hh], it & 1, ab, 93 + t))) break;
            tc_fence_after();
            issue_o_half(t, st, hh, (it > 0 || hh > 0) ? 1u : 0u);
            mma_commit(&s.o_done[t][hh]);
            if (more) {
              if (!k_next) {
                if (!(ok = mbar_wait(&s.k_full[st1], ph1, ab, 96))) break;
                tc_fence_after();
                k_next = true;
              }
              issue_s_half(t, st1, hh);
              mma_commit(&s.sh_full[t][hh]);
            }
          }
        }
        if (!ok) break;
        mma_commit(&s.v_empty[st]);
        if (more) mma_commit(&s.k_empty[st1]);
      }
      for (int it = 0; !kHalfPipe && ok && it < n_active; ++it) {
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const int st1 = (it + 1) & 1;
        const uint32_t ph1 = ((it + 1) >> 1) & 1;
        const bool more = it + 1 < n_active;
        if (!(ok = mbar_wait(&s.v_full[st], ph, ab, 92))) break;
        if (!(ok = mbar_wait(&s.p_full[0], it & 1, ab, 93))) break;
        tc_fence_after();
        issue_o(0, st, it > 0);
        if (more) {
          if (!(ok = mbar_wait(&s.k_full[st1], ph1, ab, 94))) break;
          tc_fence_after();
          issue_s(0, st1);
          mma_commit(&s.s_full[0]);
        }
        if (!(ok = mbar_wait(&s.p_full[1], it & 1, ab, 95))) break;
        tc_fence_after();
        issue_o(1, st, it > 0);
        mma_commit(&s.v_empty[st]);
        if (more) {
          issue_s(1, st1);
          mma_commit(&s.s_full[1]);
          mma_commit(&s.k_empty[st1]);
        }
      }
      if (ok) mma_commit(&s.o_full);
      // Drain: every issued MMA has finished before TMEM is released.
      mma_commit(&s.drain);
      volatile uint32_t never = 0;
      AbortState drain_ab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.drain, 0, drain_ab, 0);
    }
  } else if (warp >= 10) {
    // ------------------------------------------------------------ ring push
    if (p.push.enabled)
      ring_push_warp(p.push, p.consume, p.status, p.wait_limit_ns, &s.abort_flag, s.trace,
                     int(warp) - 10);
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;                // query tile within the CTA
    const int qt = qt0 + t;
    const int r = threadIdx.x & 127;        // row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + t * 128;
    const uint32_t o_addr = tmem + lane_off + kOCol + t * kD;
    const bool q_valid_tile = qt < p.n_q_tiles;
    const int q_tile_pos = t == 0 ? q_pos0 : q_pos1;
    const int q_pos = q_tile_pos + r;
    // key tiles [0, full_hi) need no mask for this query tile
    int full_hi = p.n_kv_tiles - ragged;
    if (p.causal) {
      const int f = visible_prefix(p.kv_tile_pos, n_active, q_tile_pos - (kTile - 1));
      full_hi = f < full_hi ? f : full_hi;
    }
    if (!q_valid_tile) full_hi = 0;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // ---- half-tile pipeline: 64 keys per step, slot hh of this tile's columns
    for (int it = 0; kHalfPipe && !skip_compute && it < n_active; ++it) {
      const bool full = it < full_hi;  // warp-uniform
      int n_vis = 128;
      if (!full) {  // diagonal / ragged / invisible tile: this row's visible keys
        n_vis = p.sk - it * kTile;
        if (p.causal) {
          const int lim = q_pos - __ldg(p.kv_tile_pos + it) + 1;
          n_vis = lim < n_vis ? lim : n_vis;
        }
        if (!q_valid_tile) n_vis = 0;
      }
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int kidx = 2 * it + hh;  // PV_t steps so far
        ok = __all_sync(0xffffffffu, mbar_wait(&s.sh_full[t][hh], it & 1, ab, 20 + t));
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld32(s_addr + hh * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld32(s_addr + hh * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_wait_ld();
        regs_defined32(&sr[0]);
        regs_defined32(&sr[32]);
        if (!full) {
          const int nv = n_vis - hh * 64;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= nv) sr[c] = 0xff800000u;  // -inf
        }
        const float tmax = row_max<64>(sr) * p.scale_log2;
        const float m_new = fmaxf(m, tmax);
        float alpha = 1.f;
        bool rescale = false;
        if (kidx == 0) {
          m = m_new;
        } else if (m_new > m + kRescaleThreshold) {
          alpha = ex2_approx(m - m_new);
          m = m_new;
          rescale = true;
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        float lacc[4] = {0.f, 0.f, 0.f, 0.f}, unused[4];
        uint32_t pk[32];
        exp_pairs<kF16, 0, true, 32>(sr, 0, p.scale_log2, neg_m, pk, lacc, unused);
        tmem_st32(s_addr + hh * 64, pk);
        // O may only be rescaled once PV_t of the previous half step has
        // finished (o_done[t][hh ^ 1], phase `it` after half 0, `it - 1` after
        // half 1). The wait runs at every step, so every phase of both barriers
        // is waited for in order and the parity never aliases.
        const bool resc = __any_sync(0xffffffffu, rescale);
        if (kidx > 0) {
          const uint32_t par = uint32_t(hh ? it : it - 1) & 1u;
          ok = __all_sync(0xffffffffu, mbar_wait(&s.o_done[t][hh ^ 1], par, ab, 24 + t));
          if (!ok) break;
        }
        if (resc) {
          tc_fence_after();
#pragma unroll
          for (int ch = 0; ch < kOChunks; ++ch) {
            uint32_t orow[32];
            tmem_ld32(o_addr + ch * 32, orow);
            tmem_wait_ld();
            regs_defined32(orow);
#pragma unroll
            for (int c = 0; c < 32; ++c)
              orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
            tmem_st32(o_addr + ch * 32, orow);
            tmem_wait_st();
            regs_live32(orow);
          }
        }
        tmem_wait_st();
        regs_live32(pk);
        tc_fence_before();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.ph_full[t][hh]);
        l = l * alpha + ((lacc[0] + lacc[1]) + (lacc[2] + lacc[3]));
      }
      if (!ok) break;
    }
    // ---- whole-tile pipeline
    for (int it = 0; !kHalfPipe && !skip_compute && it < n_active; ++it) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[t], it & 1, ab, 20 + t));
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
      tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
      const bool full = it < full_hi;  // warp-uniform
      int n_vis = 128;
      if (!full) {  // diagonal / ragged / invisible tile: count this row's visible keys
        n_vis = p.sk - it * kTile;
        if (p.causal) {
          const int lim = q_pos - __ldg(p.kv_tile_pos + it) + 1;
          n_vis = lim < n_vis ? lim : n_vis;
        }
        if (!q_valid_tile) n_vis = 0;
      }
      tmem_wait_ld();
      regs_defined32(&sr[0]);
      regs_defined32(&sr[32]);
      regs_defined32(&sr[64]);
      regs_defined32(&sr[96]);
      if (!full) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= n_vis) sr[c] = 0xff800000u;  // -inf
      }
      // row max of the raw scores (scale > 0 commutes with max)
      float mx0 = __uint_as_float(sr[0]), mx1 = __uint_as_float(sr[1]);
      float mx2 = __uint_as_float(sr[2]), mx3 = __uint_as_float(sr[3]);
#pragma unroll
      for (int c = 4; c < 128; c += 8) {
        mx0 = max3f(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mx1 = max3f(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = max3f(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = max3f(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      const float tmax = fmaxf(max3f(mx0, mx1, mx2), mx3) * p.scale_log2;
      const float m_new = fmaxf(m, tmax);
      float alpha = 1.f;
      bool rescale = false;
      if (it == 0) {
        m = m_new;
      } else if (m_new > m + kRescaleThreshold) {
        alpha = ex2_approx(m - m_new);
        m = m_new;
        rescale = true;
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      l *= alpha;
      const float neg_m = -m_use;
      uint32_t pk[2][32];
      if constexpr (kPackedExp) {
        // f32x2 arithmetic: one FMA and one add instruction per pair of scores
        float lacc[4] = {0.f, 0.f, 0.f, 0.f};
        exp_half<kF16, 0, true>(sr, 0, p.scale_log2, neg_m, pk[0], lacc);
        tmem_st32(s_addr, pk[0]);
        exp_half<kF16, 0, true>(sr, 1, p.scale_log2, neg_m, pk[1], lacc);
        tmem_st32(s_addr + 32, pk[1]);
        l += (lacc[0] + lacc[1]) + (lacc[2] + lacc[3]);
      } else {
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const int c = half * 32 + cc;
            const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * c]), p.scale_log2, neg_m));
            const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * c + 1]), p.scale_log2, neg_m));
            if (c & 1) { l2 += p0; l3 += p1; } else { l0 += p0; l1 += p1; }
            pk[half][cc] = pack16<kF16>(p0, p1);
          }
          tmem_st32(s_addr + half * 32, pk[half]);
        }
        l += (l0 + l1) + (l2 + l3);
      }
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int ch = 0; ch < kOChunks; ++ch) {
          uint32_t orow[32];
          tmem_ld32(o_addr + ch * 32, orow);
          tmem_wait_ld();
          regs_defined32(orow);
#pragma unroll
          for (int c = 0; c < 32; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
          tmem_st32(o_addr + ch * 32, orow);
          tmem_wait_st();
          regs_live32(orow);
        }
      }
      tmem_wait_st();
      regs_live32(pk[0]);
      regs_live32(pk[1]);
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&s.p_full[t]);
    }
    if (!skip_compute && ok) ok = __all_sync(0xffffffffu, mbar_wait(&s.o_full, 0, ab, 30 + t));
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (p.trace && threadIdx.x == 0) s.trace[3] = globaltimer();

    // ---- epilogue: normalise, merge with the running state, store
    // Everything above only read q and this step's K/V; the running state was
    // written by the previous step's grid, which must be complete from here on.
    if (p.dependent_launch) asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = qt * kTile + r;
    const bool row_valid = qt < p.n_q_tiles && row < p.sq;
    const float lse2_new = (l > 0.f) ? m + log2f(l) : -INFINITY;
    const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
    float w_prev = 0.f, w_new = 1.f, lse2 = lse2_new;
    float* lse_ptr = p.lse + (int64_t(b) * p.hq + h) * p.sq + (row_valid ? row : 0);
    const int64_t o_off = int64_t(b) * p.o_batch_stride + int64_t(row_valid ? row : 0) * p.o_row_stride +
                          int64_t(h) * kD;
    if (has_prior && row_valid) {
      const float lse2_prev = *lse_ptr * 1.4426950408889634f;
      const float mx = fmaxf(lse2_prev, lse2_new);
      if (mx == -INFINITY) {
        w_prev = 0.f;
        w_new = 0.f;
        lse2 = -INFINITY;
      } else {
        w_prev = ex2_approx(lse2_prev - mx);
        w_new = ex2_approx(lse2_new - mx);
        const float tot = w_prev + w_new;
        w_prev /= tot;
        w_new /= tot;
        lse2 = mx + log2f(tot);
      }
    }
    const float scale_new = w_new * inv_l;
#pragma unroll
    for (int ch = 0; ch < kOChunks; ++ch) {
      uint32_t orow[32];
      if (!skip_compute && ok) {
        tmem_ld32(o_addr + ch * 32, orow);
        tmem_wait_ld();
        regs_defined32(orow);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) orow[c] = 0u;
      }
      if (!row_valid || !ok) continue;
      float v[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(orow[c]) * scale_new;
      if (has_prior) {
        const float4* prev = reinterpret_cast<const float4*>(p.o_state + o_off + ch * 32);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float4 pv = prev[q4];
          v[4 * q4 + 0] += w_prev * pv.x;
          v[4 * q4 + 1] += w_prev * pv.y;
          v[4 * q4 + 2] += w_prev * pv.z;
          v[4 * q4 + 3] += w_prev * pv.w;
        }
      }
      if (p.final_out) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + o_off + ch * 32);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8)
          dst[q8] = make_uint4(pack16<kF16>(v[8 * q8 + 0], v[8 * q8 + 1]),
                               pack16<kF16>(v[8 * q8 + 2], v[8 * q8 + 3]),
                               pack16<kF16>(v[8 * q8 + 4], v[8 * q8 + 5]),
                               pack16<kF16>(v[8 * q8 + 6], v[8 * q8 + 7]));
      } else {
        float4* dst = reinterpret_cast<float4*>(p.o_state + o_off + ch * 32);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          dst[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
      }
    }
    if (row_valid && ok) *lse_ptr = lse2 * 0.6931471805599453f;
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc<512>(tmem);
  if (p.trace && threadIdx.x == 0) {
    const uint32_t linear_cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    s.trace[0] = (uint64_t(sm_id()) << 32) | linear_cta;
    s.trace[6] = globaltimer();
    s.trace[7] = uint64_t(n_active);
    uint64_t* dst = p.trace + uint64_t(linear_cta) * kTraceWords;
    for (int i = 0; i < kTraceWords; ++i) dst[i] = s.trace[i];
  }
  if (p.consume.enabled && p.consume.done_counter && threadIdx.x == 0) {
    // The last CTA to finish tells the left neighbour this slot may be reused
    // (without a done counter a separate signal kernel releases the slot).
    __threadfence();
    const uint32_t prev = atomicAdd(p.consume.done_counter, 1u);
    if (prev == p.consume.done_target) {
      // Every CTA has finished reading the slot: rearm the local counters, then
      // hand the slot back to the left neighbour.
      *p.consume.done_counter = 0u;
      if (p.consume.reset_arrivals) *p.consume.arrivals = 0u;
      fence_sys();
      st_release_sys(p.consume.left_credit, p.consume.left_credit_value);
    }
  }
}

// ------------------------------------------------------------------ host side
}  // namespace

CUtensorMap make_bshd_map_dt(const void* base, int64_t B, int64_t S, int64_t H, int64_t stride_b,
                             int64_t stride_s, int64_t stride_h, int D, bool fp16) {
  const uint64_t dims[4] = {uint64_t(D), uint64_t(H), uint64_t(S), uint64_t(B)};
  const uint64_t strides[3] = {uint64_t(stride_h) * 2, uint64_t(stride_s) * 2,
                               uint64_t(stride_b) * 2};
  const uint32_t box[4] = {64, 1, kTile, 1};
  return host::make_bf16_map(base, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                             fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                  : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
}

CUtensorMap make_bshd_map(const void* base, int64_t B, int64_t S, int64_t H, int64_t stride_b,
                          int64_t stride_s, int64_t stride_h) {
  return make_bshd_map_dt(base, B, S, H, stride_b, stride_s, stride_h, 128, false);
}

size_t flash_fwd_smem_bytes() { return sizeof(FwdSmem<128>) + 1024; }

namespace {
using FwdKernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                             const FwdParams);
struct FwdVariant {
  FwdKernelFn fn;
  int smem;
};
template <int kD, bool kF16>
FwdVariant fwd_variant_d(int var) {
  constexpr int smem = int(sizeof(FwdSmem<kD>) + 1024);
  switch (var) {
    case 0: return FwdVariant{flash_fwd_kernel<kD, kF16, 0>, smem};
    case 1: return FwdVariant{flash_fwd_kernel<kD, kF16, 1>, smem};
    default: return FwdVariant{flash_fwd_kernel<kD, kF16, 2>, smem};
  }
}
FwdVariant fwd_variant(int head_dim, bool fp16, int var) {
  if (head_dim == 64) return fp16 ? fwd_variant_d<64, true>(var) : fwd_variant_d<64, false>(var);
  return fp16 ? fwd_variant_d<128, true>(var) : fwd_variant_d<128, false>(var);
}
// Pipeline of FwdParams::variant -1: MGFA_FWD_VARIANT (0-2), else kDefaultFwdVariant.
int default_fwd_variant() {
  static const int v = [] {
    const char* e = std::getenv("MGFA_FWD_VARIANT");
    if (e && e[0] >= '0' && e[0] <= '2' && e[1] == 0) return e[0] - '0';
    return kDefaultFwdVariant;
  }();
  return v;
}
}  // namespace

void flash_fwd_launch_maps(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                           FwdParams& p, cudaStream_t stream) {
  MGFA_CHECK(p.head_dim == 64 || p.head_dim == 128, "head_dim must be 64 or 128");
  static int attr_device[12] = {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1};
  if (p.variant < 0) p.variant = default_fwd_variant();
  MGFA_CHECK(p.variant <= 2, "forward variant must be 0, 1 or 2");
  const FwdVariant var = fwd_variant(p.head_dim, p.fp16 != 0, p.variant);
  const int vi = ((p.head_dim == 64 ? 0 : 2) + (p.fp16 ? 1 : 0)) * 3 + p.variant;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (attr_device[vi] != dev) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(var.fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        var.smem));
    attr_device[vi] = dev;
  }
  const int n_pairs = (p.n_q_tiles + 1) / 2;
  dim3 grid(n_pairs, p.hq, p.batch);
  if (p.dependent_launch) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = size_t(var.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, var.fn, mq, mk, mv, p));
  } else {
    var.fn<<<grid, kThreads, var.smem, stream>>>(mq, mk, mv, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void flash_fwd_launch(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                      FwdParams& p, cudaStream_t stream) {
  auto map = [&](const torch::Tensor& t) {
    MGFA_CHECK(t.stride(3) == 1, "head_dim must be contiguous");
    return make_bshd_map_dt(t.data_ptr(), t.size(0), t.size(1), t.size(2), t.stride(0),
                            t.stride(1), t.stride(2), p.head_dim, p.fp16 != 0);
  };
  flash_fwd_launch_maps(map(q), map(k), map(v), p, stream);
}

int flash_fwd_grid_ctas(int hq, int n_q_tiles, int batch) {
  return hq * ((n_q_tiles + 1) / 2) * batch;
}

}  // namespace mgfa
