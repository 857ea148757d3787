// Self-test of the tcgen05 building blocks the attention kernels use, on one
// 128 x 128 tile:
//   C1 = A * B^T   A [128 x 64], B [128 x 64] bf16, both K-major, 128-byte
//                  swizzled tiles loaded by TMA, accumulator in TMEM (SS form)
//   C2 = A * V     A copied into TMEM as packed bf16 pairs (TS form),
//                  V [64 x 128] bf16 MN-major (N contiguous), loaded by TMA
// Both accumulators are read back with tcgen05.ld (32x32b) and stored as fp32.
#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>

#include "sm100_ptx.cuh"
#include "tma_host.hpp"

namespace mgfa {
namespace {

using namespace mgfa::dev;

struct __align__(1024) ProbeSmem {
  __nv_bfloat16 a[128 * 64];      // 16 KB, one 64-column swizzled box
  __nv_bfloat16 b[128 * 64];      // 16 KB
  __nv_bfloat16 v[2][64 * 64];    // two 64-column boxes of V, 8 KB each
  uint64_t bar_load;
  uint64_t bar_mma;
  uint32_t tmem_base;
  uint32_t abort_flag;
};

__global__ void __launch_bounds__(128, 1)
    umma_probe_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b,
                      const __grid_constant__ CUtensorMap map_v, const __nv_bfloat16* a_gmem,
                      float* c1, float* c2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  ProbeSmem& s = *reinterpret_cast<ProbeSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t warp = warp_id(), lane = lane_id(), tid = threadIdx.x;
  AbortState ab{&s.abort_flag, status, 2000000000ull};

  if (warp == 0) tmem_alloc<512>(&s.tmem_base);
  if (tid == 0) {
    s.abort_flag = 0;
    mbar_init(&s.bar_load, 1);
    mbar_init(&s.bar_mma, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t c1_col = 0, c2_col = 128, a_col = 256;

  if (tid == 0) {
    mbar_arrive_expect_tx(&s.bar_load, 2 * 128 * 64 * 2 + 2 * 64 * 64 * 2);
    tma_load_2d(s.a, &map_a, &s.bar_load, 0, 0);
    tma_load_2d(s.b, &map_b, &s.bar_load, 0, 0);
    tma_load_2d(s.v[0], &map_v, &s.bar_load, 0, 0);
    tma_load_2d(s.v[1], &map_v, &s.bar_load, 64, 0);
  }

  // A into TMEM: lane = row, column c holds elements (2c, 2c+1).
  {
    const uint32_t row = tid;
    uint32_t packed[32];
    for (int c = 0; c < 32; ++c) {
      const float lo = __bfloat162float(a_gmem[row * 64 + 2 * c]);
      const float hi = __bfloat162float(a_gmem[row * 64 + 2 * c + 1]);
      packed[c] = pack_bf16(lo, hi);
    }
    tmem_st32(tmem + ((warp * 32) << 16) + a_col, packed);
    tmem_wait_st();
    regs_live32(packed);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const bool loaded = mbar_wait(&s.bar_load, 0, ab, 1);
  if (tid == 0 && loaded) {
    const uint32_t idesc_ss = make_idesc_bf16(128, 128, 0, 0);
    const uint32_t idesc_ts = make_idesc_bf16(128, 128, 0, 1);
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ad = make_sdesc_sw128(smem_u32(s.a) + kk * 32, 16, 1024);
      const uint64_t bd = make_sdesc_sw128(smem_u32(s.b) + kk * 32, 16, 1024);
      mma_ss(tmem + c1_col, ad, bd, idesc_ss, kk > 0);
    }
    for (int kk = 0; kk < 4; ++kk) {
      // V: K = rows (16 per step, 128 B each), N halves 8 KB apart.
      const uint64_t vd = make_sdesc_sw128(smem_u32(s.v[0]) + kk * 2048, 8192, 1024);
      mma_ts(tmem + c2_col, tmem + a_col + kk * 8, vd, idesc_ts, kk > 0);
    }
    mma_commit(&s.bar_mma);
  }
  __syncwarp();
  const bool done = loaded && mbar_wait(&s.bar_mma, 0, ab, 2);
  tc_fence_after();
  if (done) {
    const uint32_t row = tid;
    for (int chunk = 0; chunk < 4; ++chunk) {
      uint32_t r[32];
      tmem_ld32(tmem + ((warp * 32) << 16) + c1_col + chunk * 32, r);
      tmem_wait_ld();
      regs_defined32(r);
      for (int j = 0; j < 32; ++j) c1[row * 128 + chunk * 32 + j] = __uint_as_float(r[j]);
      tmem_ld32(tmem + ((warp * 32) << 16) + c2_col + chunk * 32, r);
      tmem_wait_ld();
      regs_defined32(r);
      for (int j = 0; j < 32; ++j) c2[row * 128 + chunk * 32 + j] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc<512>(tmem);
}

}  // namespace

// Returns (C1, C2, status) for A [128,64], B [128,64], V [64,128] bf16 CUDA tensors.
std::vector<torch::Tensor> umma_probe(torch::Tensor a, torch::Tensor b, torch::Tensor v) {
  MGFA_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.is_contiguous(),
             "a must be a contiguous bf16 CUDA tensor");
  MGFA_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.is_contiguous(),
             "b must be a contiguous bf16 CUDA tensor");
  MGFA_CHECK(v.is_cuda() && v.scalar_type() == at::kBFloat16 && v.is_contiguous(),
             "v must be a contiguous bf16 CUDA tensor");
  MGFA_CHECK(a.size(0) == 128 && a.size(1) == 64 && b.size(0) == 128 && b.size(1) == 64 &&
              v.size(0) == 64 && v.size(1) == 128);
  auto opts = a.options().dtype(at::kFloat);
  auto c1 = torch::zeros({128, 128}, opts), c2 = torch::zeros({128, 128}, opts);
  auto status = torch::zeros({1}, a.options().dtype(at::kInt));
  const uint64_t dims_ab[2] = {64, 128}, strides_ab[1] = {128};
  const uint32_t box_ab[2] = {64, 128};
  const uint64_t dims_v[2] = {128, 64}, strides_v[1] = {256};
  const uint32_t box_v[2] = {64, 64};
  CUtensorMap ma = host::make_bf16_map(a.data_ptr(), 2, dims_ab, strides_ab, box_ab);
  CUtensorMap mb = host::make_bf16_map(b.data_ptr(), 2, dims_ab, strides_ab, box_ab);
  CUtensorMap mv = host::make_bf16_map(v.data_ptr(), 2, dims_v, strides_v, box_v);
  const size_t smem = sizeof(ProbeSmem) + 1024;
  cudaFuncSetAttribute(umma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  umma_probe_kernel<<<1, 128, smem, at::cuda::getCurrentCUDAStream()>>>(
      ma, mb, mv, reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), c1.data_ptr<float>(),
      c2.data_ptr<float>(), reinterpret_cast<uint32_t*>(status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {c1, c2, status};
}

}  // namespace mgfa
