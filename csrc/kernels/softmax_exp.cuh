// Softmax exponentials of the sm_100a attention forward kernels
// (flash_fwd_sm100.cu, attn_fwd_persistent.cu): p = 2^(s * scale - m) for the
// scores of one row held in registers, summed into the row-sum accumulators and
// packed to 16-bit pairs for the PV MMA, with a selectable share of the
// exponentials computed on the FMA pipe (exp2_poly2 in sm100_ptx.cuh) instead
// of the MUFU unit. At head_dim 128 the MUFU throughput of an SM (16 per clock)
// equals the tensor core's demand of two query tiles, so moving a quarter of
// the exponentials off it leaves the softmax slack.
#pragma once

#include "sm100_ptx.cuh"

namespace mgfa {
namespace dev {

// 2^x for one x on the FMA pipe: the method of exp2_poly2, scalar.
__device__ __forceinline__ float exp2_fma1(float x) {
  constexpr float kC0 = 9.999195933e-01f, kC1 = 6.932621598e-01f, kC2 = 2.427141368e-01f,
                  kC3 = 5.521299317e-02f, kRound = 12582912.0f;  // 1.5 * 2^23
  const float xc = fmaxf(x, -126.f);
  const float t = xc + kRound;
  const float f = xc - (t - kRound);
  const float pv = fmaf(fmaf(fmaf(kC3, f, kC2), f, kC1), f, kC0);
  return __uint_as_float(__float_as_uint(pv) + (__float_as_uint(t) << 23));
}

// Probabilities of pairs [c0, c0 + kN) of a row of kCols raw scores (pair c =
// keys 2c, 2c+1): p = 2^(s * scale - m), summed into the row-sum accumulators
// and packed to 16-bit pairs (pk[c - c0]) for the PV MMA. kPacked uses the
// f32x2 instructions (two lanes of work per instruction); kPoly8 of every 8
// pairs go through the FMA-pipe polynomial instead of MUFU.EX2 (callers pass 0
// for tiles with masked scores: the polynomial clamps -inf to 2^-126 instead of
// 0). With kMax the loop also folds kCols / kN further raw scores per pair
// into `mx` (four running maxima), so the row max is computed alongside.
template <bool kF16, int kPoly8, bool kPacked, int kN, bool kMax = false, int kCols>
__device__ __forceinline__ void exp_pairs(const uint32_t (&sr)[kCols], int c0, float scale,
                                          float neg_m, uint32_t* pk, float (&lacc)[4],
                                          float (&mx)[4]) {
  constexpr int kPer = kCols / kN;  // raw scores folded into the max per pair step
  if constexpr (kPacked) {
    const uint64_t sc2 = f2_pack(scale, scale), nm2 = f2_pack(neg_m, neg_m);
    uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int cc = 0; cc < kN; ++cc) {
      const int c = c0 + cc;
      if constexpr (kMax) {
        const float* f = reinterpret_cast<const float*>(sr) + kPer * cc;
#pragma unroll
        for (int u = 0; u < kPer; u += 2) mx[(u >> 1) & 3] = max3f(mx[(u >> 1) & 3], f[u], f[u + 1]);
      }
      const uint64_t x2 = f2_fma(
          f2_pack(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), sc2, nm2);
      uint64_t e2;
      if ((cc & 7) >= 8 - kPoly8) {
        e2 = exp2_poly2(x2);
      } else {
        float a, b;
        f2_unpack(x2, a, b);
        e2 = f2_pack(ex2_approx(a), ex2_approx(b));
      }
      if (cc & 1) acc1 = f2_add(acc1, e2);
      else acc0 = f2_add(acc0, e2);
      float e0, e1;
      f2_unpack(e2, e0, e1);
      pk[cc] = pack16<kF16>(e0, e1);
    }
    float a0, a1, b0, b1;
    f2_unpack(acc0, a0, a1);
    f2_unpack(acc1, b0, b1);
    lacc[0] += a0;
    lacc[1] += a1;
    lacc[2] += b0;
    lacc[3] += b1;
  } else {
#pragma unroll
    for (int cc = 0; cc < kN; ++cc) {
      const int c = c0 + cc;
      if constexpr (kMax) {
        const float* f = reinterpret_cast<const float*>(sr) + kPer * cc;
#pragma unroll
        for (int u = 0; u < kPer; u += 2) mx[(u >> 1) & 3] = max3f(mx[(u >> 1) & 3], f[u], f[u + 1]);
      }
      const float x0 = fmaf(__uint_as_float(sr[2 * c]), scale, neg_m);
      const float x1 = fmaf(__uint_as_float(sr[2 * c + 1]), scale, neg_m);
      float p0, p1;
      if ((cc & 7) >= 8 - kPoly8) {
        p0 = exp2_fma1(x0);
        p1 = exp2_fma1(x1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      if (cc & 1) {
        lacc[2] += p0;
        lacc[3] += p1;
      } else {
        lacc[0] += p0;
        lacc[1] += p1;
      }
      pk[cc] = pack16<kF16>(p0, p1);
    }
  }
}

// One 64-key half of a 128-score row: pairs [32 half, 32 half + 32).
template <bool kF16, int kPoly8, bool kPacked>
__device__ __forceinline__ void exp_half(const uint32_t (&sr)[128], int half, float scale,
                                         float neg_m, uint32_t (&pk)[32], float (&lacc)[4]) {
  float unused[4];
  exp_pairs<kF16, kPoly8, kPacked, 32, false>(sr, half * 32, scale, neg_m, pk, lacc, unused);
}

// Row max of n raw scores (n a multiple of 8) as four interleaved chains of
// three-input maxima.
template <int kN>
__device__ __forceinline__ float row_max(const uint32_t* sr) {
  float mx0 = __uint_as_float(sr[0]), mx1 = __uint_as_float(sr[1]);
  float mx2 = __uint_as_float(sr[2]), mx3 = __uint_as_float(sr[3]);
#pragma unroll
  for (int c = 4; c < kN; c += 8) {
    mx0 = max3f(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
    mx1 = max3f(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
    mx2 = max3f(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
    mx3 = max3f(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
  }
  return fmaxf(max3f(mx0, mx1, mx2), mx3);
}

}  // namespace dev
}  // namespace mgfa
