// Parameters of the sm_100a attention backward kernels.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "flash_fwd_sm100.cuh"  // RingPush / RingConsume

namespace mgfa {

// Fused ring transport of the backward pass (dK/dV kernel side): the incoming
// accumulators of the current KV owner are read from this rank's receive slot,
// this rank's contribution is added, and the sum is stored straight into the
// right neighbour's slot (or, after the last step, its home buffer) through the
// peer mapping; one release-add per CTA signals the neighbour.
struct BwdRing {
  const float* acc_in_dk = nullptr;   // incoming accumulators (local), null = zeros
  const float* acc_in_dv = nullptr;
  float* acc_out_dk = nullptr;        // destination (peer memory)
  float* acc_out_dv = nullptr;
  uint32_t* acc_arrivals = nullptr;   // right neighbour's arrival counter of the destination
  const uint32_t* acc_credit = nullptr;  // local: right's finished uses of the destination
  uint32_t acc_credit_target = 0;
  int64_t acc_out_elems = 0;          // floats at acc_out_dk / acc_out_dv; debug builds
                                      // skip (and report) a row store past them
  int enabled = 0;
};

struct BwdParams {
  int batch = 1, hq = 1, hkv = 1;
  int head_dim = 128;                  // 64 or 128
  int fp16 = 0;                        // fp16 inputs instead of bf16
  int sq = 0, sk = 0;
  int n_q_tiles = 0, n_kv_tiles = 0;
  int sq_pad = 0;                      // n_q_tiles * 128: row stride of lse2 / delta
  float scale = 0.f;                   // softmax scale
  float scale_log2 = 0.f;              // softmax scale * log2(e)
  int causal = 0;
  const int* q_tile_pos = nullptr;     // [n_q_tiles]
  const int* kv_tile_pos = nullptr;    // [n_kv_tiles]
  const float* lse2 = nullptr;         // [B, Hq, sq_pad] LSE in log2 units
  const float* delta = nullptr;        // [B, Hq, sq_pad] rowsum(dO * O)
  // fp32 gradient outputs, [B, S, H, head_dim]; accumulate adds into what is there
  float* dq = nullptr;
  float* dk = nullptr;
  float* dv = nullptr;
  int64_t dq_batch_stride = 0, dq_row_stride = 0;
  int64_t dkv_batch_stride = 0, dkv_row_stride = 0;
  int accumulate = 0;
  uint32_t* status = nullptr;
  uint64_t wait_limit_ns = 2000000000ull;
  // fused ring transport (dK/dV kernel: push K/V + move accumulators; dQ kernel:
  // release the slot through consume.done_counter / left_credit)
  RingPush push;
  RingConsume consume;
  BwdRing ring;
};

constexpr int kDkdvThreads = 256;  // 4 softmax, TMA, MMA, 2 push warps

CUtensorMap make_bshd_map(const void* base, int64_t B, int64_t S, int64_t H,
                          int64_t stride_b, int64_t stride_s, int64_t stride_h);
void flash_bwd_dq_launch(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
                         const CUtensorMap& mv, BwdParams& p, cudaStream_t stream);
void flash_bwd_dkdv_launch(const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
                           const CUtensorMap& mv, BwdParams& p, cudaStream_t stream);
// delta[b,h,i] = sum_d dO*O, lse2 = lse * log2(e); padded rows get lse2 = +inf.
void flash_bwd_preprocess_launch(const void* o, const void* dout, int64_t o_sb, int64_t o_ss,
                                 int64_t do_sb, int64_t do_ss, const float* lse, int B, int S,
                                 int H, int s_pad, float* lse2, float* delta, cudaStream_t stream,
                                 int head_dim = 128, bool fp16 = false);

}  // namespace mgfa
