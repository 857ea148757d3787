// Reduction-throughput probe for the backward design: the traffic a fused dK/dV
// kernel would add if it accumulated dQ with vector reductions. CTA
// (key tile j, head h) adds a 128 x D fp32 tile of ones into the dQ rows of every
// query tile i it sees (i >= j when causal), 16 bytes per reduction
// (atomicAdd on float4, sm_90+), as the fused kernel would after each dQ MMA.
// dq: fp32 [heads, n_q_tiles * 128, D]; after one launch every row of query
// tile i holds the number of key tiles that reached it.
#include <torch/types.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "../common/check.hpp"

namespace mgfa {
namespace {

__global__ void __launch_bounds__(256)
    red_probe_kernel(float* __restrict__ dq, int n_q_tiles, int D, int causal) {
  const int j = blockIdx.x, h = blockIdx.y;
  const int vec_per_tile = 128 * D / 4;
  float4* base = reinterpret_cast<float4*>(dq) + int64_t(h) * n_q_tiles * vec_per_tile;
  const float4 one = make_float4(1.f, 1.f, 1.f, 1.f);
  for (int i = causal ? j : 0; i < n_q_tiles; ++i) {
    float4* tile = base + int64_t(i) * vec_per_tile;
    for (int v = threadIdx.x; v < vec_per_tile; v += blockDim.x) atomicAdd(tile + v, one);
  }
}

}  // namespace

// Adds every key tile's contribution once; returns nothing (time it with events).
void red_probe(torch::Tensor dq, int64_t n_kv_tiles, bool causal) {
  MGFA_CHECK(dq.is_cuda() && dq.scalar_type() == at::kFloat && dq.is_contiguous() &&
                 dq.dim() == 3 && dq.size(1) % 128 == 0 && dq.size(2) % 4 == 0,
             "dq must be a contiguous fp32 CUDA tensor [heads, n_q_tiles*128, D]");
  const int heads = int(dq.size(0)), n_q_tiles = int(dq.size(1) / 128), D = int(dq.size(2));
  MGFA_CHECK(n_kv_tiles > 0 && n_kv_tiles <= n_q_tiles, "0 < n_kv_tiles <= n_q_tiles");
  c10::cuda::CUDAGuard guard(dq.device());
  red_probe_kernel<<<dim3(unsigned(n_kv_tiles), unsigned(heads)), 256, 0,
                     at::cuda::getCurrentCUDAStream()>>>(dq.data_ptr<float>(), n_q_tiles, D,
                                                         causal ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mgfa
