// Torch-facing entry points of the attention kernels.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>

#include "../kernels/flash_fwd_sm100.cuh"

namespace mgfa {

void flash_fwd_launch(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                      FwdParams& p, cudaStream_t stream);
size_t flash_fwd_smem_bytes();

namespace {

void check_bshd(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 4, name, " must be [batch, seq, heads, head_dim]");
  TORCH_CHECK(t.size(3) == 128, name, ": the sm_100a kernel supports head_dim 128");
  TORCH_CHECK(t.stride(3) == 1, name, " must have a contiguous head_dim");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}

const int* tile_pos_ptr(const c10::optional<torch::Tensor>& t, int n, const char* name) {
  TORCH_CHECK(t.has_value(), "causal attention needs ", name);
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous(), name,
              " must be a contiguous int32 CUDA tensor");
  TORCH_CHECK(t->numel() >= n, name, " has ", t->numel(), " entries, need ", n);
  return t->data_ptr<int>();
}

}  // namespace

// One forward pass of q against (k, v), optionally merged into a running state.
//   q [B, Sq, Hq, 128], k/v [B, Sk, Hkv, 128] bf16.
//   o       [B, Sq, Hq, 128] bf16, written when final_out.
//   o_state [B, Sq, Hq, 128] fp32 running output, read when merge, written when !final_out.
//   lse     [B, Hq, Sq] fp32, read when merge, always written.
//   q_tile_pos / kv_tile_pos: int32 global start positions of the 128-token tiles
//     (causal only).
void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> o,
               c10::optional<torch::Tensor> o_state, torch::Tensor lse, double scale, bool causal,
               c10::optional<torch::Tensor> q_tile_pos, c10::optional<torch::Tensor> kv_tile_pos,
               bool merge, bool final_out, torch::Tensor status, int64_t wait_limit_ns) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  TORCH_CHECK(k.sizes() == v.sizes() && k.strides() == v.strides(), "k and v must match");
  TORCH_CHECK(q.size(0) == k.size(0), "batch mismatch");
  const int B = int(q.size(0)), Sq = int(q.size(1)), Hq = int(q.size(2));
  const int Sk = int(k.size(1)), Hkv = int(k.size(2));
  TORCH_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() &&
                  lse.numel() == int64_t(B) * Hq * Sq,
              "lse must be a contiguous float32 [B, Hq, Sq] tensor");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
              "status must be an int32 CUDA tensor");
  c10::cuda::CUDAGuard guard(q.device());

  FwdParams p;
  p.batch = B;
  p.hq = Hq;
  p.hkv = Hkv;
  p.sq = Sq;
  p.sk = Sk;
  p.n_q_tiles = (Sq + 127) / 128;
  p.n_kv_tiles = (Sk + 127) / 128;
  p.scale_log2 = float(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  if (causal) {
    p.q_tile_pos = tile_pos_ptr(q_tile_pos, p.n_q_tiles, "q_tile_pos");
    p.kv_tile_pos = tile_pos_ptr(kv_tile_pos, p.n_kv_tiles, "kv_tile_pos");
  }
  if (final_out) {
    TORCH_CHECK(o.has_value(), "final_out needs o");
    TORCH_CHECK(o->scalar_type() == at::kBFloat16 && o->sizes() == q.sizes() && o->stride(3) == 1,
                "o must be bf16 shaped like q");
    p.o = o->data_ptr();
  } else {
    TORCH_CHECK(o_state.has_value(), "state output needs o_state");
  }
  if (merge || !final_out) {
    TORCH_CHECK(o_state.has_value() && o_state->scalar_type() == at::kFloat &&
                    o_state->sizes() == q.sizes() && o_state->is_contiguous(),
                "o_state must be a contiguous fp32 tensor shaped like q");
    p.o_state = o_state->data_ptr<float>();
  }
  if (final_out && merge) {
    TORCH_CHECK(o->stride(0) == o_state->stride(0) && o->stride(1) == o_state->stride(1) &&
                    o->stride(2) == o_state->stride(2),
                "o and o_state must share strides");
  }
  const torch::Tensor& ref = final_out ? *o : *o_state;
  p.o_batch_stride = ref.stride(0);
  p.o_row_stride = ref.stride(1);
  TORCH_CHECK(ref.stride(2) == 128, "outputs must have packed heads");
  p.lse = lse.data_ptr<float>();
  p.merge = merge ? 1 : 0;
  p.final_out = final_out ? 1 : 0;
  p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  p.wait_limit_ns = uint64_t(wait_limit_ns);
  if (Sq == 0 || B == 0) return;
  flash_fwd_launch(q, k, v, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace mgfa
