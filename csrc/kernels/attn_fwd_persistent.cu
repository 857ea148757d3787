// Persistent attention forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One launch of a grid of one CTA per SM computes a query shard against a list
// of KV segments (attn_fwd_persistent.cuh): one segment for single-GPU
// attention, the P shards of a ring for ring attention. Work items are
// (batch, head, pair of 128-row query tiles), heads slowest and the heaviest
// pair of each head first, handed out by an atomic counter as CTAs free up
// (dynamic persistent scheduling). For one item the CTA streams the visible
// key tiles of every segment in turn; the output accumulator stays in TMEM and
// the row max / row sum in registers across segments, so the result is
// normalised and written once, with no per-step merge pass (the reference
// merges partial results with a separate kernel per ring step and normalises
// on the host: ring/attention/bench/ring_attention_nccl_gpu_bench.cu:114-135,
// 398-407).
//
// Warp roles (12 warps):
//   warps 0-3   softmax + epilogue of query tile 0 (thread = row = TMEM lane)
//   warps 4-7   softmax + epilogue of query tile 1
//   warp  8     scheduler + TMA producer (Q per item, K/V tiles in a 2-stage ring)
//   warp  9     MMA issuer (one thread): S = Q K^T (SS), O += P V (TS, P in TMEM)
//   warps 10-11 ring push (ring launches only)
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,256+D) O1 after it.
// Pipeline per key tile: PV0(j) S0(j+1) PV1(j) S1(j+1), so one softmax
// warpgroup works while the tensor core runs the other tile's GEMMs. The
// default softmax uses packed f32x2 arithmetic; template variants hand P over
// in two 64-key halves (the PV MMAs on the first half start while the softmax
// warps still exponentiate the second) or run a fraction of the exponentials
// (kPoly8 of every 8 pairs, full tiles only) as a polynomial on the FMA pipe
// instead of the MUFU unit. Both measured slower under the 1 kW power cap and
// stay selectable for tuning. O is rescaled only when the running max grows by
// more than 2^8.
//
// Ring launches (PRing::enabled): segment s >= 1 sits in this rank's receive
// slot s; the producer waits (bounded, system-scope acquire) for unit
// (s, kv-head chunk) to have arrived before its first TMA load from it, and
// the push warps forward every unit to the right neighbour's slot s + 1 (plain
// 16-byte peer stores, release-add of the neighbour's arrival counter). TMA
// only ever reads this GPU's own memory and nothing uses cluster multicast.
// The grid must be co-resident (cooperative launch): push and compute of one
// rank only wait on data that other ranks' push warps produce, never on a CTA
// of their own grid that might not be running.
//
// Every wait is bounded by %globaltimer: on expiry the kernel records a status
// code, raises the CTA's abort flag, drains its in-flight TMA loads and MMAs,
// frees TMEM and returns.
#include <torch/types.h>
#include <c10/cuda/CUDAException.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "../common/check.hpp"
#include "attn_fwd_persistent.cuh"
#include "sm100_ptx.cuh"
#include "softmax_exp.cuh"

namespace mgfa {
namespace {

using namespace mgfa::dev;

constexpr int kTile = 128;
constexpr int kHalfBytes = kTile * 64 * 2;  // one 128 x 64 16-bit swizzled box
constexpr int kWarps = 12;
constexpr int kThreads = kWarps * 32;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kNoItem = 0x7fffffff;

template <int kD>
struct __align__(1024) PSmem {
  static constexpr int kHalves = kD / 64;
  uint16_t q[2][kHalves][kTile * 64];  // [query tile][d half]
  uint16_t k[2][kHalves][kTile * 64];  // [stage][d half]
  uint16_t v[2][kHalves][kTile * 64];
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2][2];  // [query tile][key half]
  uint64_t o_full[2], o_empty[2];
  uint64_t sched_full[2], sched_empty[2];
  uint64_t drain;
  int sched_item[2];
  uint32_t tmem_base;
  uint32_t abort_flag;
  uint64_t wait_ns;  // producer time spent waiting for ring arrivals (trace)
  uint32_t softmax_done;  // softmax warps that left their item loop
};

__device__ __forceinline__ uint32_t sm_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// Phase profile of the kernel variant with bit 10 of the tune word set: per CTA
// kProfWords clock64 sums, written to PFwdParams::trace ([grid][kProfWords]).
// Softmax (lane 0 of warps 0 and 4, summed): [0] waiting for S, [1] TMEM load
// of S, [2] row max, [3] first half of P (exponentials, store, hand-over),
// [4] second half of P, [5] tiles; MMA thread: [6] waiting for V, [7] for
// P half 0 of tile 0, [8] for P half 1 of tile 0, [9] for K of the next tile,
// [10] for P half 0 of tile 1, [11] for P half 1 of tile 1, [12] tiles,
// [13] cycles of the MMA thread's whole loop.
constexpr int kProfWords = 16;

struct Prof {
  unsigned long long acc[kProfWords];
};

__device__ __forceinline__ unsigned long long clk() {
  unsigned long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

struct Item {
  int b, h, hk, qt0;
};

__device__ __forceinline__ Item decode_item(const PFwdParams& p, int item) {
  const int n_pairs = (p.n_q_tiles + 1) >> 1;
  const int bh = item / n_pairs;
  Item it;
  it.qt0 = 2 * (n_pairs - 1 - (item - bh * n_pairs));  // heaviest pair of a head first
  it.b = bh / p.hq;
  it.h = bh - it.b * p.hq;
  it.hk = it.h / (p.hq / p.hkv);
  return it;
}

// Key tiles of segment s that at least one query tile of the pair can see
// (a prefix, since every layout lists its tiles in increasing position).
// Warp-cooperative: every lane of the warp must call it.
__device__ __forceinline__ int seg_active(const PFwdParams& p, int s, int max_q_pos) {
  const int n = (p.seg_len[s] + kTile - 1) / kTile;
  if (!p.causal) return n;
  return visible_prefix(p.kv_tile_pos + s * p.kv_pos_stride, n, max_q_pos + (kTile - 1));
}

__device__ __forceinline__ int pair_max_pos(const PFwdParams& p, int qt0) {
  if (!p.causal) return 0;
  const int a = __ldg(p.q_tile_pos + qt0);
  const int b = qt0 + 1 < p.n_q_tiles ? __ldg(p.q_tile_pos + qt0 + 1) : a;
  return a > b ? a : b;
}

// ------------------------------------------------------------------ ring push
// Push warp `pw` of `n_pw` copies its parts of every unit (segment s, chunk c)
// into the right neighbour's slot s + 1 and signals each part.
template <int kD>
__device__ void push_units(const PFwdParams& p, int pw, int n_pw, volatile uint32_t* abort_flag,
                           uint64_t* t_start, uint64_t* t_end) {
  const PRing& R = p.ring;
  const uint32_t lane = lane_id();
  const int n_chunks = p.batch * p.hkv;
  const int L = p.kv_rows;
  constexpr int kRowBytes = kD * 2;
  constexpr int kPieces = kRowBytes / 16;       // 16-byte pieces per row
  constexpr int kRowsPerPass = 32 / kPieces;     // rows a warp covers per instruction
  const int rows_per_part = (L + kPushUnitParts - 1) / kPushUnitParts;
  if (pw >= kPushUnitParts) return;
  // The right neighbour must have finished reading its slots in the previous call.
  bool ok = true;
  if (lane == 0) {
    ok = wait_flag_geq(R.credit, R.call, p.wait_limit_ns, p.status, 40, 0);
    if (!ok) *abort_flag = 1;
    *t_start = globaltimer();
  }
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok) return;
  const int piece = int(lane) % kPieces, sub_row = int(lane) / kPieces;
  for (int c = 0; c < n_chunks; ++c) {
    const int b = c / p.hkv, hk = c - b * p.hkv;
    for (int s = 0; s + 1 < p.n_seg; ++s) {
      if (*abort_flag) return;
      if (s >= 1) {  // the unit must have fully arrived here before we forward it
        if (lane == 0) {
          ok = wait_flag_geq(R.arrivals + s * kPMaxChunks + c, uint32_t(kPushUnitParts),
                             p.wait_limit_ns, p.status, 41, uint32_t(s));
          if (!ok) *abort_flag = 1;
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) return;
      }
      for (int part = pw; part < kPushUnitParts; part += n_pw) {
        const int r0 = part * rows_per_part;
        const int r1 = r0 + rows_per_part < L ? r0 + rows_per_part : L;
        for (int kv = 0; kv < 2; ++kv) {
          const uint8_t* src_base =
              s == 0 ? (kv == 0 ? R.own_k : R.own_v)
                     : R.slots + (uint64_t(s - 1) * 2 + kv) * R.shard_bytes;
          uint8_t* dst_base = R.peer_slots + (uint64_t(s) * 2 + kv) * R.shard_bytes;
          // rows r0.. of (b, hk): element offset ((b * L + r) * Hkv + hk) * D
          for (int r = r0 + sub_row; r < r1; r += kRowsPerPass * 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int rr = r + u * kRowsPerPass;
              if (rr < r1) {
                const uint64_t off =
                    ((uint64_t(b) * L + rr) * p.hkv + hk) * uint64_t(kRowBytes) + piece * 16;
                v[u] = *reinterpret_cast<const uint4*>(src_base + off);
              }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int rr = r + u * kRowsPerPass;
              if (rr < r1) {
                const uint64_t off =
                    ((uint64_t(b) * L + rr) * p.hkv + hk) * uint64_t(kRowBytes) + piece * 16;
                uint8_t* dst = dst_base + off;
                if (MGFA_IN_BOUNDS(!R.peer_slots_end || dst + 16 <= R.peer_slots_end, p.status,
                                   42))
                  *reinterpret_cast<uint4*>(dst) = v[u];
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          // The unit's tag goes with part 0, before its release: a consumer that
          // saw every part arrive also sees the tag.
          if (part == 0)
            *reinterpret_cast<volatile uint32_t*>(R.peer_tags + (s + 1) * kPMaxChunks + c) =
                R.seg_tag[s];
          if (!(R.drop_signal && s == 0 && c == 0 && part == 0)) {
            fence_sys();
            red_release_sys_add(R.peer_arrivals + (s + 1) * kPMaxChunks + c, 1u);
          }
        }
        __syncwarp();
      }
    }
  }
  if (lane == 0) *t_end = globaltimer();
}

// ------------------------------------------------------------------ kernel
// kVar: bit 0 packed f32x2 softmax arithmetic, bit 1 P handed over in two halves,
// bit 2 phase profile (see Prof), bit 3 row max as a shallow tree, bit 4
// speculative exponentials against the running max (the tile max is folded in
// alongside and a tile whose max grew by more than 2^8 is redone), bit 5 the
// wait for the first half's P store hidden behind the next quarter's
// exponentials.
template <int kD, bool kF16, int kPoly8, bool kRing, int kVar>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_persistent_kernel(const __grid_constant__ CUtensorMap map_q,
                               const __grid_constant__ CUtensorMap map_k,
                               const __grid_constant__ CUtensorMap map_v,
                               const __grid_constant__ CUtensorMap map_slots,
                               const __grid_constant__ PFwdParams p) {
  constexpr int kHalves = kD / 64;
  constexpr int kTileBytes = kHalves * kHalfBytes;
  constexpr int kKSteps = kD / 16;
  constexpr int kOChunks = kD / 32;
  constexpr uint32_t kOCol = 256;
  constexpr bool kPacked = (kVar & 1) != 0;
  constexpr bool kSplit = (kVar & 2) != 0;
  constexpr bool kProfile = (kVar & 4) != 0;
  constexpr bool kTreeMax = (kVar & 8) != 0;
  constexpr bool kSpec = (kVar & 16) != 0;  // speculative exponentials (running max)
  constexpr bool kLate = (kVar & 32) != 0;  // P-store wait behind the next quarter
  unsigned long long pa[kProfWords];
#pragma unroll
  for (int i = 0; i < kProfWords; ++i) pa[i] = 0;
  [[maybe_unused]] unsigned long long c0 = 0, c1 = 0;
  extern __shared__ uint8_t smem_raw[];
  PSmem<kD>& s = *reinterpret_cast<PSmem<kD>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const uint32_t warp = warp_id(), lane = lane_id();
  AbortState ab{&s.abort_flag, p.status, p.wait_limit_ns};
  uint64_t tr_start = globaltimer(), tr_push0 = 0, tr_push1 = 0;
  if (warp == 0) tmem_alloc<512>(&s.tmem_base);
  if (threadIdx.x == 0) {
    s.abort_flag = 0;
    s.wait_ns = 0;
    s.softmax_done = 0;
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i][0], 4);  // one arrive per softmax warp
      mbar_init(&s.p_full[i][1], 4);
      mbar_init(&s.o_full[i], 1);
      mbar_init(&s.o_empty[i], 4);
      mbar_init(&s.sched_full[i], 1);
      mbar_init(&s.sched_empty[i], 9);  // MMA thread + 8 softmax warps
    }
    mbar_init(&s.drain, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  int items_done = 0;

  // Push-only CTAs (PRing::push_ctas > 0): every warp pushes; these CTAs take
  // no work item, so the dynamic scheduler hands all items to the others.
  const int first_push_cta = kRing ? int(gridDim.x) - p.ring.push_ctas : int(gridDim.x);
  const bool push_cta = kRing && p.ring.push_ctas > 0 && int(blockIdx.x) >= first_push_cta;
  if (push_cta) {
    push_units<kD>(p, (int(blockIdx.x) - first_push_cta) * kWarps + int(warp),
                   p.ring.push_ctas * kWarps, &s.abort_flag, &tr_push0, &tr_push1);
  } else if (warp == 8) {
    // ------------------------------------------------------------ scheduler + TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      if (kRing) tma_prefetch_desc(&map_slots);
    }
    uint32_t it = 0;
    int n = 0;
    bool ok = true;
    int ready_chunk = -1;
    uint32_t ready_mask = 0;
    int last_k_phase[2] = {-1, -1}, last_v_phase[2] = {-1, -1}, last_q_phase = -1;
    while (true) {
      int item = kNoItem;
      if (lane == 0) {
        if (ok && !s.abort_flag) item = int(atomicAdd(p.sched, 1u));
        if (item >= p.n_items) item = kNoItem;
        const int slot = n & 1;
        if (!mbar_wait(&s.sched_empty[slot], ((n >> 1) & 1) ^ 1, ab, 80)) {
          ok = false;
          item = kNoItem;
        }
        s.sched_item[slot] = item;
        mbar_arrive(&s.sched_full[slot]);
      }
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item == kNoItem) break;
      const Item I = decode_item(p, item);
      const int max_pos = pair_max_pos(p, I.qt0);
      if (lane == 0) {
        ok = mbar_wait(&s.q_empty, (n & 1) ^ 1, ab, 81);
        if (ok) {
          mbar_arrive_expect_tx(&s.q_full, 2 * kTileBytes);
          for (int t = 0; t < 2; ++t)
            for (int hf = 0; hf < kHalves; ++hf)
              tma_load_4d(s.q[t][hf], &map_q, &s.q_full, hf * 64, I.h, (I.qt0 + t) * kTile, I.b);
          last_q_phase = n & 1;
        }
      }
      for (int sg = 0; sg < p.n_seg; ++sg) {
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        const int n_act = seg_active(p, sg, max_pos);
        if (n_act == 0) continue;
        const bool from_slot = kRing && sg >= 1;
        if (from_slot) {
          const int chunk = I.b * p.hkv + I.hk;
          if (chunk != ready_chunk) {
            ready_chunk = chunk;
            ready_mask = 0;
          }
          if (!((ready_mask >> sg) & 1u)) {
            if (lane == 0) {
              const uint64_t w0 = globaltimer();
              ok = wait_flag_geq(p.ring.arrivals + sg * kPMaxChunks + chunk,
                                 uint32_t(kPushUnitParts), p.wait_limit_ns, p.status, 8,
                                 uint32_t(sg));
              if (ok && ld_acquire_sys(p.ring.tags + sg * kPMaxChunks + chunk) !=
                            p.ring.seg_tag[sg]) {
                record_error(p.status, kErrTagMismatch, 8, uint32_t(sg));
                ok = false;
              }
              if (!ok) s.abort_flag = 1;
              s.wait_ns += globaltimer() - w0;
              // data written by peers' generic stores, read next by the async proxy
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            ready_mask |= 1u << sg;
          }
        }
        if (lane == 0) {
          const CUtensorMap* mk = from_slot ? &map_slots : &map_k;
          const CUtensorMap* mv = from_slot ? &map_slots : &map_v;
          const int ck = from_slot ? ((sg - 1) * 2 + 0) * p.batch + I.b : I.b;
          const int cv = from_slot ? ((sg - 1) * 2 + 1) * p.batch + I.b : I.b;
          for (int j = 0; ok && j < n_act; ++j) {
            const int st = int(it & 1);
            const uint32_t ph = (it >> 1) & 1;
            if (!(ok = mbar_wait(&s.k_empty[st], ph ^ 1, ab, 82))) break;
            mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
            for (int hf = 0; hf < kHalves; ++hf)
              tma_load_4d(s.k[st][hf], mk, &s.k_full[st], hf * 64, I.hk, j * kTile, ck);
            last_k_phase[st] = int(ph);
            if (!(ok = mbar_wait(&s.v_empty[st], ph ^ 1, ab, 83))) break;
            mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
            for (int hf = 0; hf < kHalves; ++hf)
              tma_load_4d(s.v[st][hf], mv, &s.v_full[st], hf * 64, I.hk, j * kTile, cv);
            last_v_phase[st] = int(ph);
            ++it;
          }
        }
        it = __shfl_sync(0xffffffffu, it, 0);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++n;
      items_done = n;
    }
    // Drain: never leave the CTA with a TMA write outstanding.
    if (lane == 0) {
      volatile uint32_t never = 0;
      AbortState drain_ab{&never, nullptr, p.wait_limit_ns};
      if (last_q_phase >= 0) mbar_wait(&s.q_full, uint32_t(last_q_phase), drain_ab, 0);
      for (int st = 0; st < 2; ++st) {
        if (last_k_phase[st] >= 0) mbar_wait(&s.k_full[st], uint32_t(last_k_phase[st]), drain_ab, 0);
        if (last_v_phase[st] >= 0) mbar_wait(&s.v_full[st], uint32_t(last_v_phase[st]), drain_ab, 0);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
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
    // half h of the 128 keys: 4 MMAs of 16 keys
    auto issue_o = [&](int t, int st, int h, bool acc) {
      const uint32_t vb = smem_u32(s.v[st][0]);
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int kk = h * 4 + k4;
        mma_ts(tmem + kOCol + t * kD, tmem + t * 128 + kk * 8,
               make_sdesc_sw128(vb + kk * 2048, kHalfBytes, 1024), idesc_o,
               (acc || kk > 0) ? 1u : 0u);
      }
    };
    uint32_t it = 0;
    int n = 0;
    bool ok = true;
    [[maybe_unused]] const unsigned long long mma_t0 = kProfile ? clk() : 0ull;
    while (true) {
      const int slot = n & 1;
      int item = kNoItem;
      if (lane == 0) {
        if (mbar_wait(&s.sched_full[slot], (n >> 1) & 1, ab, 90)) item = s.sched_item[slot];
        mbar_arrive(&s.sched_empty[slot]);
      }
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item == kNoItem) break;
      const Item I = decode_item(p, item);
      const int max_pos = pair_max_pos(p, I.qt0);
      int T = 0;
      for (int sg = 0; sg < p.n_seg; ++sg) T += seg_active(p, sg, max_pos);
      if (lane == 0) {
        ok = mbar_wait(&s.q_full, n & 1, ab, 91);
        if (ok && T == 0) {
          // No visible key tile: no MMA, but the item still takes one phase of
          // each O hand-over. Without the o_empty waits this thread would run a
          // phase ahead of a slow epilogue, whose parity wait then aliases (a
          // stall, or the next item's first PV overwriting O while the previous
          // item's epilogue still reads it).
          mma_commit(&s.q_empty);
          ok = mbar_wait(&s.o_empty[0], (n & 1) ^ 1, ab, 94) &&
               mbar_wait(&s.o_empty[1], (n & 1) ^ 1, ab, 98);
          if (ok) {
            mma_commit(&s.o_full[0]);
            mma_commit(&s.o_full[1]);
          }
        } else if (ok) {
          {
            const int st = int(it & 1);
            if ((ok = mbar_wait(&s.k_full[st], (it >> 1) & 1, ab, 92))) {
              tc_fence_after();
              issue_s(0, st);
              mma_commit(&s.s_full[0]);
              issue_s(1, st);
              mma_commit(&s.s_full[1]);
              mma_commit(&s.k_empty[st]);
              if (T == 1) mma_commit(&s.q_empty);
            }
          }
          for (int j = 0; ok && j < T; ++j) {
            const uint32_t g = it + uint32_t(j);
            const int st = int(g & 1);
            const uint32_t ph = (g >> 1) & 1, pp = g & 1;
            const int st1 = int((g + 1) & 1);
            const uint32_t ph1 = ((g + 1) >> 1) & 1;
            const bool more = j + 1 < T;
            if constexpr (kProfile) c0 = clk();
            if (!(ok = mbar_wait(&s.v_full[st], ph, ab, 93))) break;
            if constexpr (kProfile) { c1 = clk(); pa[6] += c1 - c0; c0 = c1; }
            if (j == 0 && !(ok = mbar_wait(&s.o_empty[0], (n & 1) ^ 1, ab, 94))) break;
            if (!(ok = mbar_wait(&s.p_full[0][0], pp, ab, 95))) break;
            if constexpr (kProfile) { c1 = clk(); pa[7] += c1 - c0; }
            tc_fence_after();
            issue_o(0, st, 0, j > 0);
            if constexpr (kProfile) c0 = clk();
            if (!(ok = mbar_wait(&s.p_full[0][1], pp, ab, 96))) break;
            if constexpr (kProfile) { c1 = clk(); pa[8] += c1 - c0; }
            tc_fence_after();
            issue_o(0, st, 1, true);
            if (!more) mma_commit(&s.o_full[0]);
            if (more) {
              if constexpr (kProfile) c0 = clk();
              if (!(ok = mbar_wait(&s.k_full[st1], ph1, ab, 97))) break;
              if constexpr (kProfile) { c1 = clk(); pa[9] += c1 - c0; }
              tc_fence_after();
              issue_s(0, st1);
              mma_commit(&s.s_full[0]);
            }
            if (j == 0 && !(ok = mbar_wait(&s.o_empty[1], (n & 1) ^ 1, ab, 98))) break;
            if constexpr (kProfile) c0 = clk();
            if (!(ok = mbar_wait(&s.p_full[1][0], pp, ab, 99))) break;
            if constexpr (kProfile) { c1 = clk(); pa[10] += c1 - c0; }
            tc_fence_after();
            issue_o(1, st, 0, j > 0);
            if constexpr (kProfile) c0 = clk();
            if (!(ok = mbar_wait(&s.p_full[1][1], pp, ab, 100))) break;
            if constexpr (kProfile) { c1 = clk(); pa[11] += c1 - c0; pa[12] += 1; }
            tc_fence_after();
            issue_o(1, st, 1, true);
            mma_commit(&s.v_empty[st]);
            if (!more) mma_commit(&s.o_full[1]);
            if (more) {
              issue_s(1, st1);
              mma_commit(&s.s_full[1]);
              mma_commit(&s.k_empty[st1]);
              if (j + 2 == T) mma_commit(&s.q_empty);
            }
          }
          it += uint32_t(T);
        }
      }
      it = __shfl_sync(0xffffffffu, it, 0);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++n;
      if (!ok) break;
    }
    if constexpr (kProfile) pa[13] = clk() - mma_t0;
    if (lane == 0) {
      // Drain: every issued MMA has finished before TMEM is released.
      mma_commit(&s.drain);
      volatile uint32_t never = 0;
      AbortState drain_ab{&never, nullptr, p.wait_limit_ns};
      mbar_wait(&s.drain, 0, drain_ab, 0);
    }
  } else if (warp >= 10) {
    // ------------------------------------------------------------ ring push
    if (kRing && p.ring.push_ctas == 0) {
      if (p.ring.push_after_compute) {
        // diagnostic: start pushing only once this CTA's compute is over
        volatile uint32_t* done = &s.softmax_done;
        const uint64_t t0 = globaltimer();
        while (*done < 8u && globaltimer() - t0 < p.wait_limit_ns) __nanosleep(256);
      }
      push_units<kD>(p, int(blockIdx.x) * 2 + int(warp - 10), int(gridDim.x) * 2, &s.abort_flag,
                     &tr_push0, &tr_push1);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = int(warp >> 2);  // query tile within the pair
    const int r = int(threadIdx.x & 127);
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + t * 128;
    const uint32_t o_addr = tmem + lane_off + kOCol + t * kD;
    uint32_t g = 0;
    int n = 0;
    bool ok = true;
    while (ok) {
      const int slot = n & 1;
      int item = kNoItem;
      if (lane == 0 && mbar_wait(&s.sched_full[slot], (n >> 1) & 1, ab, 20 + t))
        item = s.sched_item[slot];
      item = __shfl_sync(0xffffffffu, item, 0);
      if (lane == 0) mbar_arrive(&s.sched_empty[slot]);
      if (item == kNoItem) break;
      const Item I = decode_item(p, item);
      const int qt = I.qt0 + t;
      const bool q_valid = qt < p.n_q_tiles;
      const int q_tile_pos = p.causal ? __ldg(p.q_tile_pos + (q_valid ? qt : I.qt0)) : 0;
      const int q_pos = q_tile_pos + r;
      const int max_pos = pair_max_pos(p, I.qt0);
      float m = -INFINITY, l = 0.f;
      bool first = true;
      bool any = false;
      for (int sg = 0; ok && sg < p.n_seg; ++sg) {
        const int n_act = seg_active(p, sg, max_pos);
        if (n_act == 0) continue;
        any = true;
        const int len = p.seg_len[sg];
        const int* kpos = p.kv_tile_pos + sg * p.kv_pos_stride;
        // key tiles [0, full_hi) need no mask for this query tile
        int full_hi = (len / kTile) < n_act ? (len / kTile) : n_act;
        if (p.causal) {
          const int f = visible_prefix(kpos, n_act, q_tile_pos - (kTile - 1));
          full_hi = f < full_hi ? f : full_hi;
        }
        if (!q_valid) full_hi = 0;
        for (int j = 0; j < n_act; ++j, ++g) {
          if constexpr (kProfile) c0 = clk();
          ok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[t], g & 1, ab, 22 + t));
          if (!ok) break;
          if constexpr (kProfile) { c1 = clk(); pa[0] += c1 - c0; c0 = c1; pa[5] += 1; }
          tc_fence_after();
          uint32_t sr[128];
          tmem_ld64_sync(s_addr, sr);  // load and wait in one statement
          tmem_ld64_sync(s_addr + 64, sr + 64);
          const bool full = j < full_hi;  // warp-uniform
          int n_vis = 128;
          if (!full) {  // diagonal / ragged / invisible tile: this row's visible keys
            n_vis = len - j * kTile;
            if (p.causal) {
              const int lim = q_pos - __ldg(kpos + j) + 1;
              n_vis = lim < n_vis ? lim : n_vis;
            }
            if (!q_valid) n_vis = 0;
          }
          if constexpr (kProfile) { c1 = clk(); pa[1] += c1 - c0; c0 = c1; }
          if (!full) {
#pragma unroll
            for (int c = 0; c < 128; ++c)
              if (c >= n_vis) sr[c] = 0xff800000u;  // -inf
          }
          float alpha = 1.f;
          bool rescale = false;
          float lacc[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t pk0[32], pk1[32];
          // Speculation: the first half's exponentials use the running max
          // while the tile max is folded in alongside; a row whose max grew by
          // more than 2^8 redoes the half (rare once a row's max has settled).
          const bool spec =
              kSpec && full && !first && __all_sync(0xffffffffu, m != -INFINITY);
          if (spec) {
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            exp_pairs<kF16, kPoly8, kPacked, 32, true>(sr, 0, p.scale_log2, -m, pk0, lacc, mx);
            const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.scale_log2;
            const bool redo = tmax > m + kRescaleThreshold;
            if (__any_sync(0xffffffffu, redo)) {
              // S of the first half is still in TMEM (P has not overwritten it):
              // reload it a quarter at a time rather than keep it in registers
              if (redo) {
                alpha = ex2_approx(m - tmax);
                m = tmax;
                rescale = true;
                lacc[0] = lacc[1] = lacc[2] = lacc[3] = 0.f;
              }
              const float nm = redo ? -m : 0.f;
#pragma unroll
              for (int qq = 0; qq < 2; ++qq) {
                tmem_ld32_sync(s_addr + qq * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[qq * 32]));
                if (redo) {
                  uint32_t pq[16];
                  float unused_mx[4];
                  exp_pairs<kF16, kPoly8, kPacked, 16>(sr, qq * 16, p.scale_log2, nm, pq, lacc,
                                                       unused_mx);
#pragma unroll
                  for (int i = 0; i < 16; ++i) pk0[qq * 16 + i] = pq[i];
                }
              }
            }
            if constexpr (kProfile) { c1 = clk(); pa[2] += c1 - c0; c0 = c1; }
          } else {
            float tmax;
            if constexpr (kTreeMax) {
              // 16 independent chains of 8 scores, then a 3-level tree: the
              // dependent depth is 7 instead of 16
              float gm[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float* f = reinterpret_cast<const float*>(sr) + 8 * i;
                gm[i] = fmaxf(max3f(max3f(max3f(f[0], f[1], f[2]), f[3], f[4]), f[5], f[6]), f[7]);
              }
              const float h0 = max3f(gm[0], gm[1], gm[2]), h1 = max3f(gm[3], gm[4], gm[5]);
              const float h2 = max3f(gm[6], gm[7], gm[8]), h3 = max3f(gm[9], gm[10], gm[11]);
              const float h4 = max3f(gm[12], gm[13], gm[14]);
              tmax = max3f(max3f(h0, h1, h2), max3f(h3, h4, gm[15]), h0) * p.scale_log2;
            } else {
              float mx0 = __uint_as_float(sr[0]), mx1 = __uint_as_float(sr[1]);
              float mx2 = __uint_as_float(sr[2]), mx3 = __uint_as_float(sr[3]);
#pragma unroll
              for (int c = 4; c < 128; c += 8) {
                mx0 = max3f(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
                mx1 = max3f(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
                mx2 = max3f(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
                mx3 = max3f(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
              }
              tmax = fmaxf(max3f(mx0, mx1, mx2), mx3) * p.scale_log2;
            }
            const float m_new = fmaxf(m, tmax);
            if (first) {
              m = m_new;
            } else if (m_new > m + kRescaleThreshold) {
              alpha = ex2_approx(m - m_new);
              m = m_new;
              rescale = true;
            }
            if constexpr (kProfile) { c1 = clk(); pa[2] += c1 - c0; c0 = c1; }
            const float m0 = (m == -INFINITY) ? 0.f : m;
            if (kPoly8 > 0 && full) exp_half<kF16, kPoly8, kPacked>(sr, 0, p.scale_log2, -m0, pk0, lacc);
            else exp_half<kF16, 0, kPacked>(sr, 0, p.scale_log2, -m0, pk0, lacc);
          }
          first = false;
          const float m_use = (m == -INFINITY) ? 0.f : m;
          // O already holds the previous tiles' PV (their MMAs completed before
          // this tile's S was committed) and must be rescaled before this tile's
          // PV starts. Rare: without a rescale the first half of P goes to the
          // tensor core while the second is computed; with one, O is rescaled
          // once the scores are no longer needed (register pressure) and both
          // halves are released together.
          const bool resc = __any_sync(0xffffffffu, rescale);
          const bool early = kSplit && !resc;
          float unused[4];
          if (early) {
            tmem_st32(s_addr, pk0);
            if constexpr (kLate) {
              // the store's completion wait goes behind a quarter of the
              // second half's exponentials
              if (kPoly8 > 0 && full)
                exp_pairs<kF16, kPoly8, kPacked, 16>(sr, 32, p.scale_log2, -m_use, pk1, lacc, unused);
              else
                exp_pairs<kF16, 0, kPacked, 16>(sr, 32, p.scale_log2, -m_use, pk1, lacc, unused);
            }
            tmem_wait_st();
            regs_live32(pk0);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.p_full[t][0]);
          }
          if constexpr (kProfile) { c1 = clk(); pa[3] += c1 - c0; c0 = c1; }
          if (kLate && early) {
            if (kPoly8 > 0 && full)
              exp_pairs<kF16, kPoly8, kPacked, 16>(sr, 48, p.scale_log2, -m_use, pk1 + 16, lacc, unused);
            else
              exp_pairs<kF16, 0, kPacked, 16>(sr, 48, p.scale_log2, -m_use, pk1 + 16, lacc, unused);
          } else {
            if (kPoly8 > 0 && full) exp_half<kF16, kPoly8, kPacked>(sr, 1, p.scale_log2, -m_use, pk1, lacc);
            else exp_half<kF16, 0, kPacked>(sr, 1, p.scale_log2, -m_use, pk1, lacc);
          }
          if (resc) {
#pragma unroll
            for (int ch = 0; ch < kOChunks; ++ch) {
              uint32_t orow[32];
              tmem_ld32_sync(o_addr + ch * 32, orow);
#pragma unroll
              for (int c = 0; c < 32; ++c)
                orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
              tmem_st32_sync(o_addr + ch * 32, orow);
            }
          }
          if (early) {
            tmem_st32_sync(s_addr + 32, pk1);
          } else {
            tmem_st32x2_sync(s_addr, pk0, pk1);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (!early) mbar_arrive(&s.p_full[t][0]);
            mbar_arrive(&s.p_full[t][1]);
          }
          if constexpr (kProfile) { c1 = clk(); pa[4] += c1 - c0; }
          l = l * alpha + ((lacc[0] + lacc[1]) + (lacc[2] + lacc[3]));
        }
      }
      if (!ok) break;
      // ---- epilogue: wait for the last PV, read O out of TMEM, free it for the
      // next item's PV, then normalise and store
      ok = __all_sync(0xffffffffu, mbar_wait(&s.o_full[t], n & 1, ab, 30 + t));
      if (!ok) break;
      tc_fence_after();
      // O goes out of TMEM in 32-column chunks; once the last chunk is loaded the
      // columns are free for the next item's PV while the stores drain.
      const int row = qt * kTile + r;
      const bool row_ok = q_valid && row < p.sq;
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      const int64_t o_off = int64_t(I.b) * p.o_batch_stride +
                            int64_t(row_ok ? row : 0) * p.o_row_stride + int64_t(I.h) * kD;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + o_off);
#pragma unroll
      for (int ch = 0; ch < kOChunks; ++ch) {
        uint32_t o[32];
        if (any) {
          tmem_ld32_sync(o_addr + ch * 32, o);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (ch == kOChunks - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.o_empty[t]);
        }
        if (row_ok) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            const float* f = reinterpret_cast<const float*>(o) + 8 * q8;
            dst[ch * 4 + q8] = make_uint4(pack16<kF16>(f[0] * inv_l, f[1] * inv_l),
                                          pack16<kF16>(f[2] * inv_l, f[3] * inv_l),
                                          pack16<kF16>(f[4] * inv_l, f[5] * inv_l),
                                          pack16<kF16>(f[6] * inv_l, f[7] * inv_l));
          }
        }
      }
      if (row_ok) {
        const float lse2 = (l > 0.f) ? m + log2f(l) : -INFINITY;
        p.lse[(int64_t(I.b) * p.hq + I.h) * p.sq + row] = lse2 * 0.6931471805599453f;
      }
      ++n;
    }
    __syncwarp();
    if (lane == 0) atomicAdd(&s.softmax_done, 1u);
  }

  // ---- teardown
  if constexpr (kProfile) {
    // softmax lane 0 of warps 0 and 4 and the MMA thread add their sums
    if (p.trace && lane == 0 && (warp == 0 || warp == 4 || warp == 9)) {
      unsigned long long* dst =
          reinterpret_cast<unsigned long long*>(p.trace) + uint64_t(blockIdx.x) * kProfWords;
      for (int i = 0; i < kProfWords; ++i)
        if (pa[i]) atomicAdd(dst + i, pa[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc<512>(tmem);
  if (warp >= 10 && lane == 0 && p.trace && kRing) {
    uint64_t* tr = p.trace + uint64_t(blockIdx.x) * kPTraceWords;
    if (warp == 10) {  // (in a push-only CTA: warp 10's own push times)
      tr[6] = tr_push0;
      tr[7] = tr_push1;
    }
  }
  if (warp == 8 && lane == 0 && p.trace && !kProfile) {
    uint64_t* tr = p.trace + uint64_t(blockIdx.x) * kPTraceWords;
    tr[0] = (uint64_t(sm_id()) << 32) | blockIdx.x;
    tr[1] = tr_start;
    tr[2] = globaltimer();
    tr[3] = uint64_t(items_done);
    tr[4] = s.wait_ns;
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.sched + 1, 1u);
    if (prev == gridDim.x - 1) {
      // Last CTA of this rank: every item was handed out and every CTA is done.
      if (kRing) {
        // Every unit of this call has to have arrived (units nobody here needed
        // too) before the counters are re-armed and the left neighbour may
        // write the slots again.
        const int n_chunks = p.batch * p.hkv;
        bool all = !s.abort_flag;
        for (int sg = 1; all && sg < p.n_seg; ++sg)
          for (int c = 0; all && c < n_chunks; ++c)
            all = wait_flag_geq(p.ring.arrivals + sg * kPMaxChunks + c,
                                uint32_t(kPushUnitParts), p.wait_limit_ns, p.status, 50,
                                uint32_t(sg));
        if (all) {
          for (int sg = 1; sg < p.n_seg; ++sg)
            for (int c = 0; c < n_chunks; ++c) p.ring.arrivals[sg * kPMaxChunks + c] = 0u;
          fence_sys();
          st_release_sys(p.ring.left_credit, p.ring.call + 1);
        }
      }
      p.sched[0] = 0u;
      p.sched[1] = 0u;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ host side
template <int kD>
constexpr int smem_bytes() {
  return int(sizeof(PSmem<kD>)) + 1024;
}

// Diagnostic switch: an environment variable set to "0".
bool getenv_flag_off(const char* name) {
  const char* v = std::getenv(name);
  return v && v[0] == '0' && v[1] == 0;
}

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const CUtensorMap, const PFwdParams);

constexpr int kDefaultPoly8 = 0;
constexpr int kDefaultVar = 1;

// poly8 / variant tuning space (head_dim 128 bf16 without the ring); every
// other combination runs the defaults.
template <int kPoly8>
KernelFn pick_var(int var) {
  switch (var) {
    case 0: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 0>;
    case 1: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 1>;
    case 2: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 2>;
    case 4: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 4>;
    case 5: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 5>;
    case 7: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 7>;
    case 11: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 11>;
    case 15: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 15>;
    case 27: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 27>;
    case 31: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 31>;
    case 43: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 43>;
    case 59: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 59>;
    case 63: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 63>;
    default: return attn_fwd_persistent_kernel<128, false, kPoly8, false, 3>;
  }
}

template <int kD, bool kF16, bool kRing>
KernelFn pick_poly(int poly8, int var) {
  if constexpr (kD == 128 && !kF16 && !kRing) {
    if (poly8 == 0) return pick_var<0>(var);
    if (poly8 == 4) return pick_var<4>(var);
    if (poly8 == 2) return pick_var<2>(var);
  }
  if constexpr (kD == 128 && !kF16 && kRing) {
    if (poly8 == 0 && var == 1) return attn_fwd_persistent_kernel<128, false, 0, true, 1>;
    if (poly8 == 0 && var == 3) return attn_fwd_persistent_kernel<128, false, 0, true, 3>;
    if (poly8 == 2 && var == 1) return attn_fwd_persistent_kernel<128, false, 2, true, 1>;
  }
  return attn_fwd_persistent_kernel<kD, kF16, kDefaultPoly8, kRing, kDefaultVar>;
}

template <int kD>
KernelFn pick(bool fp16, bool ring, int poly8, int var) {
  if (ring)
    return fp16 ? pick_poly<kD, true, true>(poly8, var) : pick_poly<kD, false, true>(poly8, var);
  return fp16 ? pick_poly<kD, true, false>(poly8, var) : pick_poly<kD, false, false>(poly8, var);
}

}  // namespace

int attn_fwd_persistent_smem_bytes(int head_dim) {
  return head_dim == 64 ? smem_bytes<64>() : smem_bytes<128>();
}

void attn_fwd_persistent_launch(const CUtensorMap& mq, const CUtensorMap& mk,
                                const CUtensorMap& mv, const CUtensorMap& mslots, int head_dim,
                                bool fp16, PFwdParams& p, int grid, int tune,
                                cudaStream_t stream) {
  MGFA_CHECK(head_dim == 64 || head_dim == 128, "head_dim must be 64 or 128");
  MGFA_CHECK(p.n_seg >= 1 && p.n_seg <= kPMaxSeg, "segment count out of range");
  MGFA_CHECK(p.sched != nullptr, "the persistent forward needs its work counters");
  MGFA_CHECK(!p.ring.enabled || p.batch * p.hkv <= kPMaxChunks, "too many kv-head chunks");
  const bool ring = p.ring.enabled != 0;
  const int var = tune < 0 ? kDefaultVar : (tune >> 8) & 63;
  const int poly8 = tune < 0 ? -1 : tune & 0xff;
  const KernelFn fn =
      head_dim == 64 ? pick<64>(fp16, ring, poly8, var) : pick<128>(fp16, ring, poly8, var);
  const int smem = attn_fwd_persistent_smem_bytes(head_dim);
  {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> ready;  // (kernel, device) with the attribute set
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (ready.insert({reinterpret_cast<const void*>(fn), dev}).second)
      C10_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  // Ring launches wait on data pushed by other ranks' grids while pushing their
  // own: every CTA must be resident at once.
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ring && !getenv_flag_off("MGFA_P_COOP") ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, fn, mq, mk, mv, mslots, p));
}

}  // namespace mgfa
