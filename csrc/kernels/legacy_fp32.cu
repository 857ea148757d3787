// fp32 SIMT attention kernels for the reference-compatible numerics path.
//
// The reference computes one partial attention of a query block against one KV
// shard (two passes over the keys, atomicAdd into the output, no scale,
// K == V), merges it into a running (m, l, acc) with a second kernel and
// normalises on the host (ring/attention/bench/ring_attention_nccl_gpu_bench.cu:
// 47-135, 398-407). These kernels produce the same quantities in one pass:
//   legacy_partial: one thread per (query row, head); keys stream through
//     shared memory 32 at a time; online softmax in fp32; optional softmax
//     scale, separate K and V, GQA and a causal mask from global token
//     positions. With `merge` set it starts from the running state and writes
//     the merged state back (no separate merge kernel needed).
//   legacy_merge:   the reference's merge (scale each side by exp(m_i - max)).
//   legacy_normalize: acc / l on the device.
#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>

#include <cfloat>
#include <cmath>

namespace mgfa {
namespace {

constexpr int kD = 64;
constexpr int kRows = 128;   // threads (query rows) per CTA
constexpr int kKeys = 32;    // keys per shared-memory tile

__global__ void __launch_bounds__(kRows)
    legacy_partial_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                          const float* __restrict__ V, int sq, int sk, int hq, int hkv,
                          float scale, const int64_t* __restrict__ q_pos,
                          const int64_t* __restrict__ k_pos, int causal, float* __restrict__ acc,
                          float* __restrict__ m_io, float* __restrict__ l_io, int merge) {
  __shared__ float ks[kKeys][kD];
  __shared__ float vs[kKeys][kD];
  const int h = blockIdx.y;
  const int hk = h / (hq / hkv);
  const int row = blockIdx.x * kRows + threadIdx.x;
  const bool valid = row < sq;

  float q[kD], o[kD];
  float m = -INFINITY, l = 0.f;
  const int64_t qoff = (int64_t(row) * hq + h) * kD;
  const int64_t ml_off = int64_t(h) * sq + row;
#pragma unroll
  for (int d = 0; d < kD; ++d) {
    q[d] = valid ? Q[qoff + d] * scale : 0.f;
    o[d] = 0.f;
  }
  if (valid && merge) {
    m = m_io[ml_off];
    l = l_io[ml_off];
#pragma unroll
    for (int d = 0; d < kD; ++d) o[d] = acc[qoff + d];
  }
  const int64_t my_pos = (causal && valid) ? q_pos[row] : 0;

  for (int k0 = 0; k0 < sk; k0 += kKeys) {
    __syncthreads();
    for (int e = threadIdx.x; e < kKeys * kD; e += kRows) {
      const int kr = e / kD, d = e % kD;
      const int key = k0 + kr;
      const int64_t off = (int64_t(key) * hkv + hk) * kD + d;
      ks[kr][d] = key < sk ? K[off] : 0.f;
      vs[kr][d] = key < sk ? V[off] : 0.f;
    }
    __syncthreads();
    float sc[kKeys];
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      const int key = k0 + j;
      bool vis = key < sk;
      if (causal && vis) vis = k_pos[key] <= my_pos;
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < kD; ++d) dot += q[d] * ks[j][d];
      sc[j] = vis ? dot : -INFINITY;
      tmax = fmaxf(tmax, sc[j]);
    }
    const float m_new = fmaxf(m, tmax);
    if (m_new == -INFINITY) continue;  // nothing visible yet
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
    m = m_new;
    l *= alpha;
#pragma unroll
    for (int d = 0; d < kD; ++d) o[d] *= alpha;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      const float pj = expf(sc[j] - m);
      l += pj;
#pragma unroll
      for (int d = 0; d < kD; ++d) o[d] += pj * vs[j][d];
    }
  }
  if (!valid) return;
  m_io[ml_off] = m;
  l_io[ml_off] = l;
#pragma unroll
  for (int d = 0; d < kD; ++d) acc[qoff + d] = o[d];
}

__global__ void legacy_merge_kernel(float* __restrict__ m_run, float* __restrict__ l_run,
                                    float* __restrict__ acc_run, const float* __restrict__ m_new,
                                    const float* __restrict__ l_new,
                                    const float* __restrict__ acc_new, int sq, int hq) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (head, row) flattened [hq, sq]
  if (i >= sq * hq) return;
  const int h = i / sq, row = i % sq;
  const float mo = m_run[i], mn = m_new[i];
  const float mx = fmaxf(mo, mn);
  const float so = (mo == -INFINITY) ? 0.f : expf(mo - mx);
  const float sn = (mn == -INFINITY) ? 0.f : expf(mn - mx);
  const int64_t off = (int64_t(row) * hq + h) * kD;
  for (int d = 0; d < kD; ++d) acc_run[off + d] = so * acc_run[off + d] + sn * acc_new[off + d];
  l_run[i] = so * l_run[i] + sn * l_new[i];
  m_run[i] = mx;
}

__global__ void legacy_normalize_kernel(const float* __restrict__ acc, const float* __restrict__ l,
                                        float* __restrict__ out, float* __restrict__ lse,
                                        const float* __restrict__ m, int sq, int hq) {
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= int64_t(sq) * hq * kD) return;
  const int64_t rh = e / kD;  // row * hq + h
  const int h = int(rh % hq), row = int(rh / hq);
  const float lv = l[int64_t(h) * sq + row];
  out[e] = lv > 0.f ? acc[e] / lv : 0.f;
  if (lse && (e % kD) == 0)
    lse[int64_t(h) * sq + row] = lv > 0.f ? m[int64_t(h) * sq + row] + logf(lv) : -INFINITY;
}

void check_f32(const torch::Tensor& t, const char* name) {
  MGFA_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), name,
              " must be a contiguous float32 CUDA tensor");
}

}  // namespace

// Q [sq, hq, 64], K/V [sk, hkv, 64]; acc [sq, hq, 64], m/l [hq, sq].
void legacy_partial(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos,
                    bool causal, torch::Tensor acc, torch::Tensor m, torch::Tensor l,
                    bool merge) {
  check_f32(q, "q");
  check_f32(k, "k");
  check_f32(v, "v");
  check_f32(acc, "acc");
  check_f32(m, "m");
  check_f32(l, "l");
  MGFA_CHECK(q.dim() == 3 && q.size(2) == kD && k.size(2) == kD && v.size(2) == kD,
              "legacy kernels need head_dim 64");
  const int sq = int(q.size(0)), hq = int(q.size(1)), sk = int(k.size(0)), hkv = int(k.size(1));
  MGFA_CHECK(hq % hkv == 0, "query heads must be a multiple of kv heads");
  const int64_t* qp = nullptr;
  const int64_t* kp = nullptr;
  if (causal) {
    MGFA_CHECK(q_pos.has_value() && k_pos.has_value(), "causal needs q_pos and k_pos");
    MGFA_CHECK(q_pos->scalar_type() == at::kLong && k_pos->scalar_type() == at::kLong,
               "positions must be int64");
    MGFA_CHECK(q_pos->numel() >= sq && k_pos->numel() >= sk, "too few positions");
    qp = q_pos->data_ptr<int64_t>();
    kp = k_pos->data_ptr<int64_t>();
  }
  if (sq == 0) return;
  dim3 grid((sq + kRows - 1) / kRows, hq);
  legacy_partial_kernel<<<grid, kRows, 0, at::cuda::getCurrentCUDAStream()>>>(
      q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), sq, sk, hq, hkv,
      float(scale), qp, kp, causal ? 1 : 0, acc.data_ptr<float>(), m.data_ptr<float>(),
      l.data_ptr<float>(), merge ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void legacy_merge(torch::Tensor m_run, torch::Tensor l_run, torch::Tensor acc_run,
                  torch::Tensor m_new, torch::Tensor l_new, torch::Tensor acc_new) {
  for (auto* t : {&m_run, &l_run, &acc_run, &m_new, &l_new, &acc_new}) check_f32(*t, "state");
  const int hq = int(acc_run.size(1)), sq = int(acc_run.size(0));
  const int n = sq * hq;
  if (n == 0) return;
  legacy_merge_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      m_run.data_ptr<float>(), l_run.data_ptr<float>(), acc_run.data_ptr<float>(),
      m_new.data_ptr<float>(), l_new.data_ptr<float>(), acc_new.data_ptr<float>(), sq, hq);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void legacy_normalize(torch::Tensor acc, torch::Tensor l, torch::Tensor out,
                      c10::optional<torch::Tensor> lse, c10::optional<torch::Tensor> m) {
  check_f32(acc, "acc");
  check_f32(l, "l");
  check_f32(out, "out");
  const int sq = int(acc.size(0)), hq = int(acc.size(1));
  const int64_t n = int64_t(sq) * hq * kD;
  if (n == 0) return;
  float* lse_p = nullptr;
  const float* m_p = nullptr;
  if (lse.has_value()) {
    MGFA_CHECK(m.has_value(), "lse output needs m");
    lse_p = lse->data_ptr<float>();
    m_p = m->data_ptr<float>();
  }
  legacy_normalize_kernel<<<int((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc.data_ptr<float>(), l.data_ptr<float>(), out.data_ptr<float>(), lse_p, m_p, sq, hq);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mgfa
