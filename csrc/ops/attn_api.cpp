// Torch-facing entry points of the attention kernels.
#include <torch/types.h>
#include "../common/check.hpp"
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>

#include "../kernels/flash_fwd_sm100.cuh"

namespace mgfa {

void flash_fwd_launch(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                      FwdParams& p, cudaStream_t stream);
size_t flash_fwd_smem_bytes();

namespace {

// bf16 / fp16 [B, S, H, D] CUDA tensor with D in `dims` and a contiguous head_dim.
void check_bshd_dims(const torch::Tensor& t, const char* name, std::initializer_list<int> dims) {
  MGFA_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  MGFA_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, name,
              " must be bfloat16 or float16");
  MGFA_CHECK(t.dim() == 4, name, " must be [batch, seq, heads, head_dim]");
  bool ok = false;
  for (int d : dims) ok = ok || t.size(3) == d;
  MGFA_CHECK(ok, name, ": unsupported head_dim ", t.size(3));
  MGFA_CHECK(t.stride(3) == 1, name, " must have a contiguous head_dim");
  MGFA_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}

void check_bshd(const torch::Tensor& t, const char* name) { check_bshd_dims(t, name, {64, 128}); }

void check_same_kind(const torch::Tensor& a, const torch::Tensor& b, const char* what) {
  MGFA_CHECK(a.scalar_type() == b.scalar_type() && a.size(3) == b.size(3), what,
              ": dtype and head_dim must match");
}

const int* tile_pos_ptr(const c10::optional<torch::Tensor>& t, int n, const char* name) {
  MGFA_CHECK(t.has_value(), "causal attention needs ", name);
  MGFA_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous(), name,
              " must be a contiguous int32 CUDA tensor");
  MGFA_CHECK(t->numel() >= n, name, " has ", t->numel(), " entries, need ", n);
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
               bool merge, bool final_out, torch::Tensor status, int64_t wait_limit_ns,
               int64_t variant) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  MGFA_CHECK(k.sizes() == v.sizes() && k.strides() == v.strides(), "k and v must match");
  check_same_kind(q, k, "q/k");
  check_same_kind(q, v, "q/v");
  MGFA_CHECK(q.size(0) == k.size(0), "batch mismatch");
  const int B = int(q.size(0)), Sq = int(q.size(1)), Hq = int(q.size(2));
  const int Sk = int(k.size(1)), Hkv = int(k.size(2));
  MGFA_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
  MGFA_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() &&
                  lse.numel() == int64_t(B) * Hq * Sq,
              "lse must be a contiguous float32 [B, Hq, Sq] tensor");
  MGFA_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
              "status must be an int32 CUDA tensor");
  c10::cuda::CUDAGuard guard(q.device());

  FwdParams p;
  p.head_dim = int(q.size(3));
  p.fp16 = q.scalar_type() == at::kHalf ? 1 : 0;
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
    MGFA_CHECK(o.has_value(), "final_out needs o");
    MGFA_CHECK(o->scalar_type() == q.scalar_type() && o->sizes() == q.sizes() &&
                    o->stride(3) == 1,
                "o must have q's dtype and shape");
    p.o = o->data_ptr();
  } else {
    MGFA_CHECK(o_state.has_value(), "state output needs o_state");
  }
  if (merge || !final_out) {
    MGFA_CHECK(o_state.has_value() && o_state->scalar_type() == at::kFloat &&
                    o_state->sizes() == q.sizes() && o_state->is_contiguous(),
                "o_state must be a contiguous fp32 tensor shaped like q");
    p.o_state = o_state->data_ptr<float>();
  }
  if (final_out && merge) {
    MGFA_CHECK(o->stride(0) == o_state->stride(0) && o->stride(1) == o_state->stride(1) &&
                    o->stride(2) == o_state->stride(2),
                "o and o_state must share strides");
  }
  const torch::Tensor& ref = final_out ? *o : *o_state;
  p.o_batch_stride = ref.stride(0);
  p.o_row_stride = ref.stride(1);
  MGFA_CHECK(ref.stride(2) == q.size(3), "outputs must have packed heads");
  p.lse = lse.data_ptr<float>();
  p.merge = merge ? 1 : 0;
  p.final_out = final_out ? 1 : 0;
  p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  p.wait_limit_ns = uint64_t(wait_limit_ns);
  MGFA_CHECK(variant >= -1 && variant <= 2, "variant must be -1, 0, 1 or 2");
  p.variant = int(variant);
  if (Sq == 0 || B == 0) return;
  flash_fwd_launch(q, k, v, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace mgfa

// ---------------------------------------------------------------------- backward
#include "../kernels/flash_bwd_sm100.cuh"

namespace mgfa {

// Gradients of one attention pass (fp32 accumulators, [B,S,H,128]).
//   dout, out: [B,Sq,Hq,128] bf16; lse [B,Hq,Sq] fp32 (of the FULL attention).
//   With accumulate the results are added to dq / dk / dv.
//   lse2 / delta: optional precomputed [B,Hq,ceil(Sq/128)*128] fp32 buffers
//   (flash_bwd_preprocess); computed here when absent.
void flash_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
               torch::Tensor out, torch::Tensor lse, torch::Tensor dq, torch::Tensor dk,
               torch::Tensor dv, double scale, bool causal,
               c10::optional<torch::Tensor> q_tile_pos, c10::optional<torch::Tensor> kv_tile_pos,
               bool accumulate, c10::optional<torch::Tensor> lse2_in,
               c10::optional<torch::Tensor> delta_in, torch::Tensor status,
               int64_t wait_limit_ns) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  check_bshd(dout, "dout");
  check_bshd(out, "out");
  MGFA_CHECK(dout.sizes() == q.sizes() && out.sizes() == q.sizes(), "dout/out must match q");
  check_same_kind(q, k, "q/k");
  check_same_kind(q, v, "q/v");
  check_same_kind(q, dout, "q/dout");
  check_same_kind(q, out, "q/out");
  const int D = int(q.size(3));
  const bool f16 = q.scalar_type() == at::kHalf;
  MGFA_CHECK(k.sizes() == v.sizes() && k.strides() == v.strides(), "k and v must match");
  const int B = int(q.size(0)), Sq = int(q.size(1)), Hq = int(q.size(2));
  const int Sk = int(k.size(1)), Hkv = int(k.size(2));
  MGFA_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
  for (auto* t : {&dq, &dk, &dv})
    MGFA_CHECK(t->scalar_type() == at::kFloat && t->dim() == 4 && t->stride(3) == 1 &&
                    t->stride(2) == q.size(3),
                "gradient buffers must be fp32 [B,S,H,D] with packed heads");
  MGFA_CHECK(dk.strides() == dv.strides(), "dk and dv must share strides");
  MGFA_CHECK(dq.sizes() == q.sizes() && dk.sizes() == k.sizes() && dv.sizes() == v.sizes(),
              "gradient buffers must match their inputs");
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int n_q_tiles = (Sq + 127) / 128, sq_pad = n_q_tiles * 128;
  torch::Tensor lse2, delta;
  if (lse2_in.has_value() && delta_in.has_value()) {
    lse2 = *lse2_in;
    delta = *delta_in;
    MGFA_CHECK(lse2.numel() == int64_t(B) * Hq * sq_pad && delta.numel() == lse2.numel(),
                "lse2/delta must be [B, Hq, ceil(Sq/128)*128]");
  } else {
    lse2 = torch::empty({B, Hq, sq_pad}, q.options().dtype(at::kFloat));
    delta = torch::empty({B, Hq, sq_pad}, q.options().dtype(at::kFloat));
    flash_bwd_preprocess_launch(out.data_ptr(), dout.data_ptr(), out.stride(0), out.stride(1),
                                dout.stride(0), dout.stride(1), lse.data_ptr<float>(), B, Sq, Hq,
                                sq_pad, lse2.data_ptr<float>(), delta.data_ptr<float>(), stream, D,
                                f16);
  }
  BwdParams p;
  p.head_dim = D;
  p.fp16 = f16 ? 1 : 0;
  p.batch = B;
  p.hq = Hq;
  p.hkv = Hkv;
  p.sq = Sq;
  p.sk = Sk;
  p.n_q_tiles = n_q_tiles;
  p.n_kv_tiles = (Sk + 127) / 128;
  p.sq_pad = sq_pad;
  p.scale = float(scale);
  p.scale_log2 = float(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  if (causal) {
    p.q_tile_pos = tile_pos_ptr(q_tile_pos, p.n_q_tiles, "q_tile_pos");
    p.kv_tile_pos = tile_pos_ptr(kv_tile_pos, p.n_kv_tiles, "kv_tile_pos");
  }
  p.lse2 = lse2.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dk = dk.data_ptr<float>();
  p.dv = dv.data_ptr<float>();
  p.dq_batch_stride = dq.stride(0);
  p.dq_row_stride = dq.stride(1);
  p.dkv_batch_stride = dk.stride(0);
  p.dkv_row_stride = dk.stride(1);
  p.accumulate = accumulate ? 1 : 0;
  p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  p.wait_limit_ns = uint64_t(wait_limit_ns);
  if (B == 0 || Sq == 0 || Sk == 0) return;
  auto map = [&](const torch::Tensor& t) {
    return make_bshd_map_dt(t.data_ptr(), t.size(0), t.size(1), t.size(2), t.stride(0),
                            t.stride(1), t.stride(2), D, f16);
  };
  const CUtensorMap mq = map(q), mdo = map(dout), mk = map(k), mv = map(v);
  flash_bwd_dkdv_launch(mq, mdo, mk, mv, p, stream);
  flash_bwd_dq_launch(mq, mdo, mk, mv, p, stream);
}

// lse2 = lse * log2(e) (+inf for rows without keys), delta = rowsum(dout * out), both
// [B, Hq, ceil(Sq/128)*128].
std::vector<torch::Tensor> flash_bwd_preprocess(torch::Tensor dout, torch::Tensor out,
                                                torch::Tensor lse) {
  check_bshd(dout, "dout");
  check_bshd(out, "out");
  const int B = int(out.size(0)), Sq = int(out.size(1)), Hq = int(out.size(2));
  const int sq_pad = (Sq + 127) / 128 * 128;
  c10::cuda::CUDAGuard guard(out.device());
  auto lse2 = torch::empty({B, Hq, sq_pad}, out.options().dtype(at::kFloat));
  auto delta = torch::empty({B, Hq, sq_pad}, out.options().dtype(at::kFloat));
  flash_bwd_preprocess_launch(out.data_ptr(), dout.data_ptr(), out.stride(0), out.stride(1),
                              dout.stride(0), dout.stride(1), lse.data_ptr<float>(), B, Sq, Hq,
                              sq_pad, lse2.data_ptr<float>(), delta.data_ptr<float>(),
                              at::cuda::getCurrentCUDAStream(), int(out.size(3)),
                              out.scalar_type() == at::kHalf);
  return {lse2, delta};
}

}  // namespace mgfa

namespace mgfa {

// Failure-path check: one forward launch whose KV "arrival" flag is a local word
// that nothing ever sets. The producer's bounded wait must expire after
// wait_limit_ns, record kErrPeerTimeout in the status word and end the kernel
// cleanly (no hang, no fault). Returns the status word (int32 CUDA tensor):
// `status` when given (so a test can aim the error at a caller's word), else a
// fresh one.
torch::Tensor fwd_timeout_probe(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                int64_t wait_limit_ns, c10::optional<torch::Tensor> status_in) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  c10::cuda::CUDAGuard guard(q.device());
  auto flags = torch::zeros({64}, q.options().dtype(at::kInt));
  torch::Tensor status;
  if (status_in.has_value()) {
    status = *status_in;
    MGFA_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
               "status must be an int32 CUDA tensor");
  } else {
    status = torch::zeros({1}, q.options().dtype(at::kInt));
  }
  auto o = torch::empty_like(q);
  auto lse = torch::empty({q.size(0), q.size(2), q.size(1)}, q.options().dtype(at::kFloat));
  FwdParams p;
  p.head_dim = int(q.size(3));
  p.fp16 = q.scalar_type() == at::kHalf ? 1 : 0;
  p.batch = int(q.size(0));
  p.hq = int(q.size(2));
  p.hkv = int(k.size(2));
  p.sq = int(q.size(1));
  p.sk = int(k.size(1));
  p.n_q_tiles = (p.sq + 127) / 128;
  p.n_kv_tiles = (p.sk + 127) / 128;
  p.scale_log2 = 0.1f;
  p.o = o.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.o_batch_stride = q.stride(0);
  p.o_row_stride = q.stride(1);
  p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  p.wait_limit_ns = uint64_t(wait_limit_ns);
  uint32_t* f = reinterpret_cast<uint32_t*>(flags.data_ptr<int>());
  p.consume.enabled = 1;
  p.consume.arrivals = f;            // never incremented
  p.consume.arrivals_target = 1;
  p.consume.done_counter = f + 16;
  p.consume.done_target = uint32_t((p.n_q_tiles + 1) / 2 * p.hq * p.batch - 1);
  p.consume.left_credit = f + 32;
  p.consume.left_credit_value = 1;
  flash_fwd_launch(q, k, v, p, at::cuda::getCurrentCUDAStream());
  return status;
}

}  // namespace mgfa

// ---------------------------------------------------------------------- persistent forward
#include "../kernels/attn_fwd_persistent.cuh"

namespace mgfa {

CUtensorMap make_bshd_map_dt(const void* base, int64_t B, int64_t S, int64_t H, int64_t stride_b,
                             int64_t stride_s, int64_t stride_h, int D, bool fp16);

int device_sm_count(int device) {
  static int counts[64] = {};
  if (device < 0 || device >= 64) return 148;
  if (!counts[device])
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&counts[device], cudaDevAttrMultiProcessorCount, device));
  return counts[device];
}

// Single-GPU forward on the persistent kernel: o [B,Sq,Hq,D] (input dtype) and
// lse [B,Hq,Sq] fp32 are written. `sched` is an int32 CUDA tensor of at least 2
// zeros that no concurrent launch uses; the kernel leaves it zeroed. grid <= 0:
// one CTA per SM (at most one per work item). With `seg_lens` the keys are
// several segments that all read (k, v) -- segment s its first seg_lens[s] rows
// at the tile positions in row s of kv_tile_pos [n_seg, n] -- and attention
// runs over their union (the ring's compute pattern on one GPU).
void flash_fwd_persistent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                          torch::Tensor lse, double scale, bool causal,
                          c10::optional<torch::Tensor> q_tile_pos,
                          c10::optional<torch::Tensor> kv_tile_pos, torch::Tensor status,
                          int64_t wait_limit_ns, torch::Tensor sched, int64_t tune,
                          int64_t grid, std::vector<int64_t> seg_lens,
                          c10::optional<torch::Tensor> trace) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  MGFA_CHECK(k.sizes() == v.sizes() && k.strides() == v.strides(), "k and v must match");
  check_same_kind(q, k, "q/k");
  check_same_kind(q, v, "q/v");
  MGFA_CHECK(q.size(0) == k.size(0), "batch mismatch");
  const int B = int(q.size(0)), Sq = int(q.size(1)), Hq = int(q.size(2));
  const int Sk = int(k.size(1)), Hkv = int(k.size(2)), D = int(q.size(3));
  const bool f16 = q.scalar_type() == at::kHalf;
  MGFA_CHECK(Hq % Hkv == 0, "query heads must be a multiple of kv heads");
  MGFA_CHECK(o.scalar_type() == q.scalar_type() && o.sizes() == q.sizes() && o.stride(3) == 1 &&
                 o.stride(2) == D,
             "o must have q's dtype and shape, with packed heads");
  MGFA_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() &&
                 lse.numel() == int64_t(B) * Hq * Sq,
             "lse must be a contiguous float32 [B, Hq, Sq] tensor");
  MGFA_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
             "status must be an int32 CUDA tensor");
  MGFA_CHECK(sched.is_cuda() && sched.scalar_type() == at::kInt && sched.numel() >= 2,
             "sched must be an int32 CUDA tensor of at least 2 zeros");
  c10::cuda::CUDAGuard guard(q.device());
  if (Sq == 0 || B == 0) return;
  PFwdParams p;
  p.batch = B;
  p.hq = Hq;
  p.hkv = Hkv;
  p.sq = Sq;
  p.n_q_tiles = (Sq + 127) / 128;
  p.n_items = B * Hq * ((p.n_q_tiles + 1) / 2);
  if (seg_lens.empty()) seg_lens.push_back(Sk);
  MGFA_CHECK(int(seg_lens.size()) <= kPMaxSeg, "at most 16 segments");
  p.n_seg = int(seg_lens.size());
  p.kv_rows = Sk;
  for (int i = 0; i < p.n_seg; ++i) {
    MGFA_CHECK(seg_lens[i] >= 0 && seg_lens[i] <= Sk, "segment length out of range");
    p.seg_len[i] = int(seg_lens[i]);
  }
  p.scale_log2 = float(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  if (causal) {
    const int n_kv_tiles = (Sk + 127) / 128;
    p.q_tile_pos = tile_pos_ptr(q_tile_pos, p.n_q_tiles, "q_tile_pos");
    p.kv_tile_pos = tile_pos_ptr(kv_tile_pos, n_kv_tiles * p.n_seg, "kv_tile_pos");
    p.kv_pos_stride = int(kv_tile_pos->numel() / p.n_seg);
    MGFA_CHECK(p.kv_pos_stride >= n_kv_tiles, "kv_tile_pos needs a row per segment");
  }
  p.o = o.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.o_batch_stride = o.stride(0);
  p.o_row_stride = o.stride(1);
  p.status = reinterpret_cast<uint32_t*>(status.data_ptr<int>());
  p.wait_limit_ns = uint64_t(wait_limit_ns);
  p.sched = reinterpret_cast<uint32_t*>(sched.data_ptr<int>());
  if (trace.has_value()) {
    MGFA_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous(),
               "trace must be a contiguous int64 CUDA tensor");
    p.trace = reinterpret_cast<uint64_t*>(trace->data_ptr<int64_t>());
  }
  auto map = [&](const torch::Tensor& t) {
    return make_bshd_map_dt(t.data_ptr(), t.size(0), t.size(1), t.size(2), t.stride(0),
                            t.stride(1), t.stride(2), D, f16);
  };
  const CUtensorMap mq = map(q), mk = map(k), mv = map(v);
  int g = int(grid);
  if (g <= 0) g = device_sm_count(q.get_device());
  if (g > p.n_items) g = p.n_items;
  attn_fwd_persistent_launch(mq, mk, mv, mk, D, f16, p, g, int(tune),
                             at::cuda::getCurrentCUDAStream());
}

}  // namespace mgfa
