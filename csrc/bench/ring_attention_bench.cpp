// Native ring-attention benchmark: the reference's ring/attention/bench programs
// (ring_attention_{staged,staged_Isendrecv,staged_Isendrecv_overlap,cuda_aware,
// cuda_aware_Isendrecv,cuda_aware_Isendrecv_overlap,nccl}_gpu_bench.cu) as one
// executable with a --backend flag, without MPI.
//
//   torchrun --nproc-per-node N --no-python build/bin/ring_attention_bench
//       <kv_size_bytes> [warmup=10] [iters=100]
//       [--backend fused|fused_stepwise|fused_one_launch|p2p_unfused|ce_unfused|nccl|
//        staged|p2p|ce]
//       [--numerics fp32|bf16] [--init legacy|randn] [--layout contiguous|zigzag|
//       striped|scheduler] [--policy dp|lpt] [--causal] [--heads H] [--kv-heads H]
//       [--head-dim D] [--seed S] [--overlap] [--json]
//
// Shapes follow the reference: tokens per rank = kv_size / (heads * head_dim * 4),
// so the global length grows with the ranks (ring_attention_nccl_gpu_bench.cu:180-200).
//   --numerics fp32 (head_dim 64): the fp32 partial-attention / merge / normalise
//     kernels of legacy_fp32.cu; backends nccl | staged, sequential or --overlap
//     (the next shard moves while the current one is computed), and p2p | ce (the
//     shard moves through RingExchange's slots by the NVLink push kernel / the
//     copy engine; sequential order). --init legacy
//     reproduces the reference's inputs (K == V, no softmax scale) so
//     `verify_full <dir> N kv_size` checks the dumps.
//   --numerics bf16 (head_dim 64 or 128): the sm_100a kernels; fused (the engine
//     MGFA_RING_ENGINE names: stepwise by default, or one_launch),
//     fused_stepwise (one attention launch per step with the transport inside
//     it), fused_one_launch (the whole ring in one launch of the persistent
//     kernel, transport inside it), p2p_unfused (the same NVLink push transport as a separate kernel on a
//     second stream), ce_unfused (the copy engine moves the shard on a second
//     stream), nccl (attention kernel per step + NCCL send/recv on a second
//     stream) or staged (device -> host -> store -> device). The bf16 total is
//     the ring on the device; the output's download into pinned memory is
//     avg_final.
// Environment as in the reference: ATTENTION_PRINT_SHARDS=1 prints token ranges
// and per-step owners of iteration 0; ATTENTION_DUMP_OUTPUT=1 writes
// ring_output_rank<r>.bin (raw little-endian fp32 [tokens x heads x dim]).
// Timing: CUDA events on the launching stream, MAX over ranks per iteration,
// mean over the timed iterations; rank 0 prints `<backend> bench: warmup=W
// iters=I` and `avg_total=... ms avg_<COMM>=... avg_attn=... avg_merge=...
// avg_final=...` (ring_attention_nccl_gpu_bench.cu:418-435).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <torch/types.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../comm/ring_engine.hpp"
#include "../comm/ring_engine_p.hpp"
#include "../comm/ring_exchange.hpp"
#include "../common/synth.hpp"
#include "../sched/shard_plan.hpp"
#include "dist_env.hpp"

namespace mgfa {
void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> o,
               c10::optional<torch::Tensor> o_state, torch::Tensor lse, double scale, bool causal,
               c10::optional<torch::Tensor> q_tile_pos, c10::optional<torch::Tensor> kv_tile_pos,
               bool merge, bool final_out, torch::Tensor status, int64_t wait_limit_ns,
               int64_t variant);
void legacy_partial(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos,
                    bool causal, torch::Tensor acc, torch::Tensor m, torch::Tensor l, bool merge);
void legacy_merge(torch::Tensor m_run, torch::Tensor l_run, torch::Tensor acc_run,
                  torch::Tensor m_new, torch::Tensor l_new, torch::Tensor acc_new);
void legacy_normalize(torch::Tensor acc, torch::Tensor l, torch::Tensor out,
                      c10::optional<torch::Tensor> lse, c10::optional<torch::Tensor> m);
}  // namespace mgfa

using mgfa::bench::Dist;
using namespace mgfa::sched;

namespace {

constexpr int kTile = 128;
constexpr int64_t kWaitNs = 2000000000;

struct Args {
  int64_t kv_size = 0;
  bool have_size = false;
  int warmup = 10, iters = 100;
  std::string backend, numerics = "fp32", init = "legacy", layout = "contiguous", policy = "lpt";
  bool causal = false, overlap = false, json = false;
  int heads = 1, kv_heads = 0, head_dim = 0;
  uint64_t seed = 0;
  int print_tables = 0;  // > 0: print the layout tables for that many ranks and exit
};

bool parse(int argc, char** argv, Args* a) {
  int pos = 0;
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto val = [&](std::string* out) {
      if (i + 1 >= argc) return false;
      *out = argv[++i];
      return true;
    };
    std::string v;
    if (s == "--backend") { if (!val(&a->backend)) return false; }
    else if (s == "--numerics") { if (!val(&a->numerics)) return false; }
    else if (s == "--init") { if (!val(&a->init)) return false; }
    else if (s == "--layout") { if (!val(&a->layout)) return false; }
    else if (s == "--policy") { if (!val(&a->policy)) return false; }
    else if (s == "--heads") { if (!val(&v)) return false; a->heads = std::atoi(v.c_str()); }
    else if (s == "--kv-heads") { if (!val(&v)) return false; a->kv_heads = std::atoi(v.c_str()); }
    else if (s == "--head-dim") { if (!val(&v)) return false; a->head_dim = std::atoi(v.c_str()); }
    else if (s == "--seed") { if (!val(&v)) return false; a->seed = uint64_t(std::atoll(v.c_str())); }
    else if (s == "--print-tables") { if (!val(&v)) return false; a->print_tables = std::atoi(v.c_str()); }
    else if (s == "--causal") a->causal = true;
    else if (s == "--overlap") a->overlap = true;
    else if (s == "--json") a->json = true;
    else if (!s.empty() && s[0] == '-') return false;
    else {
      if (pos == 0) { a->kv_size = std::atoll(s.c_str()); a->have_size = true; }
      else if (pos == 1) a->warmup = std::atoi(s.c_str());
      else if (pos == 2) a->iters = std::atoi(s.c_str());
      else return false;
      ++pos;
    }
  }
  if (a->backend.empty()) a->backend = a->numerics == "bf16" ? "fused" : "nccl";
  return (a->numerics == "fp32" || a->numerics == "bf16") &&
         (a->backend == "fused" || a->backend == "fused_stepwise" ||
          a->backend == "fused_one_launch" ||
          a->backend == "p2p_unfused" || a->backend == "ce_unfused" ||
          a->backend == "nccl" || a->backend == "staged" || a->backend == "p2p" ||
          a->backend == "ce") &&
         (a->init == "legacy" || a->init == "randn");
}

// ----------------------------------------------------------------- layout metadata
// Tile tables of the kernels, as the Python layer builds them
// (multi_gpu_flashattention_b200/parallel/layouts.py).
struct Meta {
  ShardPlan plan;
  std::string kind;
  int64_t L = 0;  // padded local length (max over ranks)

  std::vector<int> tile_starts(int rank) const {
    const int64_t n = (L + kTile - 1) / kTile;
    std::vector<int> out;
    if (kind == "striped") {
      for (int64_t t = 0; t < n; ++t) out.push_back(int(t * kTile));
      return out;
    }
    for (int64_t s : plan.tile_starts(rank, kTile)) {
      if (s < 0) throw std::runtime_error(kind + " layout: a 128-token tile is not consecutive");
      out.push_back(int(s));
    }
    while (int64_t(out.size()) < n) out.push_back(1 << 30);  // padding tiles see nothing
    for (size_t i = 1; i < out.size(); ++i)
      if (out[i] < out[i - 1]) throw std::runtime_error("tile positions must be non-decreasing");
    return out;
  }
  std::vector<int> kv_tile_pos(int rank, int owner) const {
    if (kind != "striped") return tile_starts(owner);
    std::vector<int> out = tile_starts(rank);
    for (auto& x : out) x += owner > rank ? 1 : 0;
    return out;
  }
  std::vector<int64_t> q_positions(int rank) const {
    std::vector<int64_t> out;
    if (kind == "striped") {
      for (int64_t i = 0; i < L; ++i) out.push_back(i);
      return out;
    }
    out = plan.positions(rank);
    while (int64_t(out.size()) < L) out.push_back(int64_t(1) << 40);
    return out;
  }
  std::vector<int64_t> k_positions(int rank, int owner) const {
    std::vector<int64_t> out;
    if (kind == "striped") {
      for (int64_t i = 0; i < L; ++i) out.push_back(i + (owner > rank ? 1 : 0));
      return out;
    }
    out = plan.positions(owner);
    while (int64_t(out.size()) < L) out.push_back(int64_t(1) << 41);
    return out;
  }
};

Meta make_meta(const Args& a, int64_t seq, int world) {
  Meta m;
  m.kind = a.layout;
  if (a.layout == "contiguous") m.plan = make_contiguous(seq, world);
  else if (a.layout == "zigzag") m.plan = make_zigzag(seq, world);
  else if (a.layout == "striped") m.plan = make_striped(seq, world);
  else if (a.layout == "scheduler")
    m.plan = make_scheduled(seq, world, kTile, a.causal ? MaskKind::Causal : MaskKind::Full,
                            a.policy);
  else throw std::runtime_error("unknown layout " + a.layout);
  m.L = m.plan.max_local_len();
  return m;
}

torch::Tensor i32_dev(const std::vector<int>& v, int dev) {
  return torch::tensor(std::vector<int32_t>(v.begin(), v.end()), torch::kInt32)
      .to(torch::Device(torch::kCUDA, dev));
}

torch::Tensor i64_dev(const std::vector<int64_t>& v, int dev) {
  return torch::tensor(v, torch::kInt64).to(torch::Device(torch::kCUDA, dev));
}

// ----------------------------------------------------------------- inputs
// Seeded N(0,1) rows (the Python layer's fill_randn_rows): out[i, :] holds
// elements [rows[i] * row_elems, (rows[i] + 1) * row_elems) of `stream`.
torch::Tensor randn_rows(uint64_t seed, uint64_t stream, const std::vector<int64_t>& rows,
                         int64_t L, int64_t row_elems) {
  auto out = torch::zeros({L, row_elems}, torch::kFloat32);
  float* p = out.data_ptr<float>();
  const int64_t n = int64_t(rows.size());
  const int nt = int(std::max(1u, std::min(32u, std::thread::hardware_concurrency())));
  std::vector<std::thread> pool;
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([=]() {
      for (int64_t i = t; i < n; i += nt)
        for (int64_t j = 0; j < row_elems; ++j)
          p[i * row_elems + j] = float(mgfa::synth::randn(
              seed, stream, uint64_t(rows[size_t(i)] * row_elems + j)));
    });
  for (auto& th : pool) th.join();
  return out;
}

// Measured sustained bf16 tensor peak (TFLOP/s) from MEASURED_PEAKS.json in the
// working directory, else 1400.
double sustained_peak_tflops() {
  FILE* f = std::fopen("MEASURED_PEAKS.json", "r");
  if (!f) return 1400.0;
  std::string text;
  char buf[4096];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, n);
  std::fclose(f);
  const std::string key = "\"bf16_tflops_sustained\"";
  const size_t at = text.find(key);
  if (at == std::string::npos) return 1400.0;
  const size_t colon = text.find(':', at + key.size());
  return colon == std::string::npos ? 1400.0 : std::atof(text.c_str() + colon + 1);
}

// ----------------------------------------------------------------- timing helpers
struct Ev {
  cudaEvent_t e;
  Ev() { cudaEventCreate(&e); }
  ~Ev() { cudaEventDestroy(e); }
  void record(cudaStream_t s) { cudaEventRecord(e, s); }
};
float elapsed(const Ev& a, const Ev& b) {
  cudaEventSynchronize(b.e);
  float ms = 0;
  cudaEventElapsedTime(&ms, a.e, b.e);
  return ms;
}

struct StepTimes {
  double total = 0, comm = 0, attn = 0, merge = 0, final = 0;
  torch::Tensor host;  // normalised output, fp32 [L, H, D]
};

// ----------------------------------------------------------------- fp32 ring
class Fp32Ring {
 public:
  Fp32Ring(const Args& a, Dist& d, const Meta& m, torch::Tensor q, torch::Tensor k,
           torch::Tensor v, double scale)
      : a_(a), d_(d), m_(m), q_(q), k_(k), v_(v), scale_(scale) {
    same_kv_ = k.data_ptr() == v.data_ptr();
    const int64_t L = q.size(0), H = q.size(1), D = q.size(2);
    auto f = torch::TensorOptions().dtype(torch::kFloat32).device(q.device());
    m_run_ = torch::empty({H, L}, f);
    l_run_ = torch::empty({H, L}, f);
    acc_run_ = torch::empty({L, H, D}, f);
    m_loc_ = torch::empty({H, L}, f);
    l_loc_ = torch::empty({H, L}, f);
    acc_loc_ = torch::empty({L, H, D}, f);
    out_ = torch::empty({L, H, D}, f);
    for (int i = 0; i < 2; ++i) {
      bufs_[i] = torch::empty_like(k);
      nbufs_[i] = torch::empty_like(v);
    }
    const int r = d.rank(), P = d.world();
    q_pos_ = i64_dev(m.q_positions(r), d.device());
    for (int o = 0; o < P; ++o) k_pos_.push_back(i64_dev(m.k_positions(r, o), d.device()));
    if (a.backend == "staged") {
      const size_t nb = size_t(k.numel()) * 4;
      for (int i = 0; i < 2; ++i) {
        cudaMallocHost(&h_send_[i], nb);
        cudaMallocHost(&h_recv_[i], nb);
      }
    }
    if (a.backend == "p2p" || a.backend == "ce") {
      // KV rotation through RingExchange's receive slots (K, then V unless K == V)
      kv_bytes_ = k.numel() * 4 * (same_kv_ ? 1 : 2);
      cudaDeviceProp prop;
      cudaGetDeviceProperties(&prop, d.device());
      ex_ = std::make_unique<mgfa::RingExchange>(d.rank(), d.world(), d.device(),
                                                 (kv_bytes_ + 4095) / 4096 * 4096,
                                                 2 * prop.multiProcessorCount);
      ex_->connect(d.all_gather(ex_->ipc_handle()));
      ex_status_ = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(
                                         torch::kCUDA, d.device()));
      cudaDeviceSynchronize();
      d.barrier();
    }
    comm_ = c10::cuda::getStreamFromPool(false, d.device());
  }
  ~Fp32Ring() {
    for (int i = 0; i < 2; ++i) {
      if (h_send_[i]) cudaFreeHost(h_send_[i]);
      if (h_recv_[i]) cudaFreeHost(h_recv_[i]);
    }
  }

  // K / V views of RingExchange slot i.
  std::array<torch::Tensor, 2> slot_kv(int i) {
    auto b = ex_->slot(i).narrow(0, 0, kv_bytes_).view(torch::kFloat32);
    const int64_t n = k_.numel();
    auto kk = b.narrow(0, 0, n).view(k_.sizes());
    return {kk, same_kv_ ? kk : b.narrow(0, n, n).view(v_.sizes())};
  }

  // Sequential ring over RingExchange: own shard, then per step one transfer into
  // slot (s+1) % 2 and the attention on it. Each push hands its slot back only
  // after reading it, and in this order every attention on a slot finishes
  // before the push that forwards (and releases) it.
  StepTimes run_exchange(bool log_steps) {
    const int P = d_.world(), r = d_.rank();
    cudaStream_t cs = at::cuda::getCurrentCUDAStream();
    StepTimes st;
    Ev t0, t1, c0, c1;
    t0.record(cs);
    c0.record(cs);
    auto own = slot_kv(0);
    own[0].copy_(k_);
    if (!same_kv_) own[1].copy_(v_);
    c1.record(cs);
    st.comm += elapsed(c0, c1);
    if (log_steps)
      std::printf("[Rank %d] step=own compute_kv_owner=%d KV tokens=%s\n", r, r,
                  m_.plan.describe(r).c_str());
    attend(k_, v_, r, true, &st);
    for (int s = 0; s < P - 1; ++s) {
      Ev s0, s1;
      s0.record(cs);
      ex_->step(s, kv_bytes_, a_.backend, ex_status_, kWaitNs);
      // the left neighbour's transfer into the slot read next may still be in flight
      ex_->wait_received(s, a_.backend, ex_status_, kWaitNs);
      s1.record(cs);
      st.comm += elapsed(s0, s1);
      const int owner = m_.plan.receive_owner(r, s);
      if (log_steps)
        std::printf("[Rank %d] step=%d received_kv_owner=%d KV tokens=%s\n", r, s, owner,
                    m_.plan.describe(owner).c_str());
      auto kv = slot_kv((s + 1) & 1);
      attend(kv[0], kv[1], owner, false, &st);
    }
    ex_->release(P - 1, a_.backend, ex_status_, kWaitNs);
    Ev f0, f1;
    f0.record(cs);
    mgfa::legacy_normalize(acc_run_, l_run_, out_, c10::nullopt, c10::nullopt);
    st.host = out_.cpu();
    f1.record(cs);
    t1.record(cs);
    cudaDeviceSynchronize();
    if (ex_status_.item<int>() != 0)
      throw std::runtime_error("transport status " + std::to_string(ex_status_.item<int>()));
    st.final = elapsed(f0, f1);
    st.total = elapsed(t0, t1);
    return st;
  }

  StepTimes run(bool log_steps) {
    if (ex_) return run_exchange(log_steps);
    const int P = d_.world(), r = d_.rank();
    cudaStream_t cs = at::cuda::getCurrentCUDAStream();
    StepTimes st;
    Ev t0, t1;
    t0.record(cs);
    torch::Tensor cur[2] = {k_, v_};
    int nxt_i = 0;
    // receive pair i: (bufs_[i], nbufs_[i]); the caller's k/v are never written
    auto nxt_of = [&](int i) { return std::array<torch::Tensor, 2>{bufs_[i], nbufs_[i]}; };
    if (!a_.overlap) {
      if (log_steps)
        std::printf("[Rank %d] step=own compute_kv_owner=%d KV tokens=%s\n", r, r,
                    m_.plan.describe(r).c_str());
      attend(cur[0], cur[1], r, true, &st);
      for (int s = 0; s < P - 1; ++s) {
        auto nxt = nxt_of(nxt_i);
        Ev c0, c1;
        c0.record(cs);
        exchange(cur, nxt.data(), cs, cs);
        c1.record(cs);
        st.comm += elapsed(c0, c1);
        const int owner = m_.plan.receive_owner(r, s);
        if (log_steps)
          std::printf("[Rank %d] step=%d received_kv_owner=%d KV tokens=%s\n", r, s, owner,
                      m_.plan.describe(owner).c_str());
        attend(nxt[0], nxt[1], owner, false, &st);
        cur[0] = nxt[0];
        cur[1] = nxt[1];
        nxt_i ^= 1;
      }
    } else {
      int owner = r;
      for (int s = 0; s < P - 1; ++s) {
        auto nxt = nxt_of(nxt_i);
        const int recv_owner = m_.plan.receive_owner(r, s);
        if (log_steps)
          std::printf("[Rank %d] step=%d compute_kv_owner=%d KV tokens=%s, receiving_kv_owner=%d "
                      "KV tokens=%s\n",
                      r, s, owner, m_.plan.describe(owner).c_str(), recv_owner,
                      m_.plan.describe(recv_owner).c_str());
        Ev ready, c0, c1;
        ready.record(cs);
        cudaStreamWaitEvent(comm_.stream(), ready.e, 0);
        c0.record(comm_.stream());
        // NCCL is asynchronous on the comm stream; the staged path blocks the
        // host, but the attention launched below was queued before it
        if (a_.backend == "nccl") exchange(cur, nxt.data(), comm_.stream(), cs);
        attend(cur[0], cur[1], owner, s == 0, &st);
        if (a_.backend == "staged") exchange(cur, nxt.data(), comm_.stream(), cs);
        c1.record(comm_.stream());
        cudaStreamWaitEvent(cs, c1.e, 0);
        cudaDeviceSynchronize();
        st.comm += elapsed(c0, c1);
        cur[0] = nxt[0];
        cur[1] = nxt[1];
        nxt_i ^= 1;
        owner = recv_owner;
      }
      if (log_steps)
        std::printf("[Rank %d] final compute_kv_owner=%d KV tokens=%s\n", r, owner,
                    m_.plan.describe(owner).c_str());
      attend(cur[0], cur[1], owner, P == 1, &st);
    }
    Ev f0, f1;
    f0.record(cs);
    mgfa::legacy_normalize(acc_run_, l_run_, out_, c10::nullopt, c10::nullopt);
    st.host = out_.cpu();
    f1.record(cs);
    t1.record(cs);
    cudaDeviceSynchronize();
    st.final = elapsed(f0, f1);
    st.total = elapsed(t0, t1);
    return st;
  }

 private:
  // Partial attention on one shard merged into the running state; synchronises
  // for the phase times, as the reference's timers do.
  void attend(const torch::Tensor& kk, const torch::Tensor& vv, int owner, bool first,
              StepTimes* st) {
    cudaStream_t cs = at::cuda::getCurrentCUDAStream();
    Ev e0, e1, e2;
    const torch::Tensor& vuse = same_kv_ ? kk : vv;
    e0.record(cs);
    mgfa::legacy_partial(q_, kk, vuse, scale_, q_pos_, k_pos_[size_t(owner)], a_.causal, acc_loc_,
                         m_loc_, l_loc_, false);
    e1.record(cs);
    if (first) {
      m_run_.copy_(m_loc_);
      l_run_.copy_(l_loc_);
      acc_run_.copy_(acc_loc_);
    } else {
      mgfa::legacy_merge(m_run_, l_run_, acc_run_, m_loc_, l_loc_, acc_loc_);
    }
    e2.record(cs);
    st->attn += elapsed(e0, e1);
    st->merge += elapsed(e1, e2);
  }

  // Moves cur -> right neighbour, left neighbour -> nxt. `s` carries the
  // transfer; `cs` is the compute stream the staged copies wait on.
  void exchange(const torch::Tensor* cur, torch::Tensor* nxt, cudaStream_t s,
                [[maybe_unused]] cudaStream_t cs) {
    const int P = d_.world(), r = d_.rank();
    const int right = (r + 1) % P, left = (r - 1 + P) % P;
    const int n_t = same_kv_ ? 1 : 2;
    const size_t nb = size_t(cur[0].numel()) * 4;
    if (a_.backend == "nccl") {
      ncclComm_t comm = d_.nccl();
      mgfa::bench::nccl_check(ncclGroupStart(), "ncclGroupStart");
      for (int i = 0; i < n_t; ++i) {
        mgfa::bench::nccl_check(ncclSend(cur[i].data_ptr(), nb, ncclUint8, right, comm, s), "ncclSend");
        mgfa::bench::nccl_check(ncclRecv(nxt[i].data_ptr(), nb, ncclUint8, left, comm, s), "ncclRecv");
      }
      mgfa::bench::nccl_check(ncclGroupEnd(), "ncclGroupEnd");
      if (s == cs) cudaStreamSynchronize(s);
    } else {
      for (int i = 0; i < n_t; ++i)
        cudaMemcpyAsync(h_send_[i], cur[i].data_ptr(), nb, cudaMemcpyDeviceToHost, s);
      cudaStreamSynchronize(s);
      for (int i = 0; i < n_t; ++i) d_.host_sendrecv(h_send_[i], nb, right, h_recv_[i], left);
      for (int i = 0; i < n_t; ++i)
        cudaMemcpyAsync(nxt[i].data_ptr(), h_recv_[i], nb, cudaMemcpyHostToDevice, s);
    }
    if (same_kv_) nxt[1] = nxt[0];
  }

  const Args& a_;
  Dist& d_;
  const Meta& m_;
  torch::Tensor q_, k_, v_;
  double scale_;
  bool same_kv_ = false;
  torch::Tensor m_run_, l_run_, acc_run_, m_loc_, l_loc_, acc_loc_, out_;
  torch::Tensor bufs_[2], nbufs_[2];
  torch::Tensor q_pos_;
  std::vector<torch::Tensor> k_pos_;
  void* h_send_[2] = {nullptr, nullptr};
  void* h_recv_[2] = {nullptr, nullptr};
  c10::cuda::CUDAStream comm_ = c10::cuda::getDefaultCUDAStream();
  std::unique_ptr<mgfa::RingExchange> ex_;
  int64_t kv_bytes_ = 0;
  torch::Tensor ex_status_;
};

// ----------------------------------------------------------------- 16-bit rings
class Bf16Ring {
 public:
  Bf16Ring(const Args& a, Dist& d, const Meta& m, torch::Tensor q, torch::Tensor k,
           torch::Tensor v, double scale)
      : a_(a), d_(d), m_(m), q_(q), k_(k), v_(v), scale_(scale) {
    const int r = d.rank(), P = d.world(), dev = d.device();
    status_ = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
    qtp_ = i32_dev(m.tile_starts(r), dev);
    std::vector<int> all;
    for (int o = 0; o < P; ++o) {
      const auto t = m.kv_tile_pos(r, o);
      all.insert(all.end(), t.begin(), t.end());
      kv_lens_.push_back(m.plan.local_len(o));
    }
    kvtp_ = i32_dev(all, dev).view({P, -1});
    const char* engine_env = std::getenv("MGFA_RING_ENGINE");
    const bool one_launch = a.backend == "fused_one_launch" ||
                            (a.backend == "fused" && engine_env &&
                             std::string(engine_env) == "one_launch");
    if (one_launch) {
      // the one-launch ring: a receive slot per step, one kernel per forward
      int64_t cap = std::max<int64_t>(k.numel() * k.element_size(), 1 << 20);
      cap = (cap + (2 << 20) - 1) / (2 << 20) * (2 << 20);
      peng_ = std::make_unique<mgfa::RingEngineP>(r, P, dev, cap);
      peng_->connect(d.all_gather(peng_->ipc_handle()));
      cudaDeviceSynchronize();
      d.barrier();
    } else if (a.backend == "fused" || a.backend == "fused_stepwise" ||
               a.backend == "p2p_unfused" || a.backend == "ce_unfused") {
      const int64_t shard = k.numel() * k.element_size();
      int64_t slot = std::max<int64_t>(shard, 1 << 20);
      slot = (slot + (2 << 20) - 1) / (2 << 20) * (2 << 20);
      const char* ch = std::getenv("MGFA_RING_CHUNKS");
      eng_ = std::make_unique<mgfa::RingEngine>(r, P, dev, slot, ch ? std::atoi(ch) : 0);
      const char* tc = std::getenv("MGFA_TAG_CHECK");
      eng_->set_tag_check(!(tc && std::string(tc) == "0"));
      const char* ca = std::getenv("MGFA_CUMULATIVE_ARRIVALS");
      eng_->set_cumulative_arrivals(!(ca && std::string(ca) == "0"));
      eng_->connect(d.all_gather(eng_->ipc_handle()));
      eng_->set_transport_mode(a.backend == "fused" || a.backend == "fused_stepwise"
                                   ? mgfa::RingEngine::kFusedPush
                               : a.backend == "p2p_unfused"  ? mgfa::RingEngine::kPushKernel
                                                             : mgfa::RingEngine::kCopyEngine);
      cudaDeviceSynchronize();
      d.barrier();
    } else {
      for (int p = 0; p < 2; ++p)
        for (int i = 0; i < 2; ++i) recv_[p][i] = torch::empty_like(i ? v : k);
      if (a.backend == "staged") {
        const size_t nb = size_t(k.numel() * k.element_size());
        for (int i = 0; i < 2; ++i) {
          cudaMallocHost(&h_send_[i], nb);
          cudaMallocHost(&h_recv_[i], nb);
        }
      } else {
        d.nccl();
      }
      comm_ = c10::cuda::getStreamFromPool(false, dev);
    }
  }
  ~Bf16Ring() {
    for (int i = 0; i < 2; ++i) {
      if (h_send_[i]) cudaFreeHost(h_send_[i]);
      if (h_recv_[i]) cudaFreeHost(h_recv_[i]);
    }
  }

  torch::Tensor status() const { return status_; }

  StepTimes run(bool log_steps) {
    const int P = d_.world(), r = d_.rank();
    if (log_steps) {
      for (int s = 0; s < P - 1; ++s) {
        const int o = m_.plan.compute_owner(r, s), ro = m_.plan.receive_owner(r, s);
        std::printf("[Rank %d] step=%d compute_kv_owner=%d KV tokens=%s, receiving_kv_owner=%d "
                    "KV tokens=%s\n",
                    r, s, o, m_.plan.describe(o).c_str(), ro, m_.plan.describe(ro).c_str());
      }
      const int o = m_.plan.compute_owner(r, P - 1);
      std::printf("[Rank %d] final compute_kv_owner=%d KV tokens=%s\n", r, o,
                  m_.plan.describe(o).c_str());
    }
    cudaStream_t cs = at::cuda::getCurrentCUDAStream();
    StepTimes st;
    // The compute-only reference (same launches, transport off) runs right
    // before and right after the ring, and the two are averaged, so clock drift
    // under the power cap does not land on one side of the comparison.
    const bool ref = (eng_ || peng_) && P > 1;
    auto compute_only = [&]() {
      Ev c0, c1;
      c0.record(cs);
      if (peng_)
        peng_->forward_compute_only(q_, k_, v_, scale_, a_.causal, opt(qtp_), opt(kvtp_),
                                    kv_lens_, status_);
      else
        eng_->forward_compute_only(q_, k_, v_, scale_, a_.causal, opt(qtp_), opt(kvtp_),
                                   kv_lens_, status_);
      c1.record(cs);
      return double(elapsed(c0, c1));
    };
    const double before = ref ? compute_only() : 0.0;
    Ev e0, e1, e2;
    e0.record(cs);
    torch::Tensor out = forward();
    e1.record(cs);
    // The output is already normalised on the device; its download into pinned
    // memory is timed on its own (avg_final), outside the ring's total.
    if (!host_out_.defined() || host_out_.sizes() != out[0].sizes())
      host_out_ = torch::empty(out[0].sizes(),
                               out.options().device(torch::kCPU).pinned_memory(true));
    host_out_.copy_(out[0], /*non_blocking=*/true);
    e2.record(cs);
    cudaDeviceSynchronize();
    st.host = host_out_.to(torch::kFloat32);
    st.total = elapsed(e0, e1);
    st.attn = elapsed(e0, e1);
    st.final = elapsed(e1, e2);
    if (ref) {
      const double comp = 0.5 * (before + compute_only());
      st.comm = std::max(0.0, st.attn - comp);  // exposed communication
      st.attn = comp;
    }
    return st;
  }

 private:
  c10::optional<torch::Tensor> opt(const torch::Tensor& t) const {
    return a_.causal ? c10::optional<torch::Tensor>(t) : c10::nullopt;
  }

  torch::Tensor forward() {
    if (peng_)
      return peng_->forward(q_, k_, v_, scale_, a_.causal, opt(qtp_), opt(kvtp_), kv_lens_,
                            status_, kWaitNs)[0];
    if (eng_)
      return eng_->forward(q_, k_, v_, scale_, a_.causal, opt(qtp_), opt(kvtp_), kv_lens_,
                           status_, kWaitNs)[0];
    const int P = d_.world(), r = d_.rank();
    const int right = (r + 1) % P, left = (r - 1 + P) % P;
    cudaStream_t cs = at::cuda::getCurrentCUDAStream();
    auto o_state = torch::empty(q_.sizes(), q_.options().dtype(torch::kFloat32));
    auto lse = torch::empty({q_.size(0), q_.size(2), q_.size(1)}, q_.options().dtype(torch::kFloat32));
    auto out = torch::empty_like(q_);
    // step t computes on cur (own k/v at t = 0, then receive pair (t-1) % 2)
    // while receive pair t % 2 fills; the caller's k/v are never written
    torch::Tensor cur[2] = {k_, v_};
    const size_t nb = size_t(k_.numel() * k_.element_size());
    for (int t = 0; t < P; ++t) {
      const int owner = (r - t + P) % P;
      const bool more = t < P - 1;
      torch::Tensor* nxt = recv_[t & 1];
      Ev ready, done;
      if (more && a_.backend == "nccl") {
        ready.record(cs);
        cudaStreamWaitEvent(comm_.stream(), ready.e, 0);
        ncclComm_t comm = d_.nccl();
        mgfa::bench::nccl_check(ncclGroupStart(), "ncclGroupStart");
        for (int i = 0; i < 2; ++i) {
          mgfa::bench::nccl_check(
              ncclSend(cur[i].data_ptr(), nb, ncclUint8, right, comm, comm_.stream()), "ncclSend");
          mgfa::bench::nccl_check(
              ncclRecv(nxt[i].data_ptr(), nb, ncclUint8, left, comm, comm_.stream()), "ncclRecv");
        }
        mgfa::bench::nccl_check(ncclGroupEnd(), "ncclGroupEnd");
        done.record(comm_.stream());
      }
      const int64_t kl = kv_lens_[size_t(owner)];
      mgfa::flash_fwd(q_, cur[0].narrow(1, 0, kl), cur[1].narrow(1, 0, kl), out, o_state, lse,
                      scale_, a_.causal, opt(qtp_),
                      a_.causal ? c10::optional<torch::Tensor>(kvtp_[owner]) : c10::nullopt,
                      t > 0, t == P - 1, status_, kWaitNs, -1);
      if (!more) break;
      if (a_.backend == "nccl") {
        cudaStreamWaitEvent(cs, done.e, 0);
      } else {
        for (int i = 0; i < 2; ++i)
          cudaMemcpyAsync(h_send_[i], cur[i].data_ptr(), nb, cudaMemcpyDeviceToHost, cs);
        cudaStreamSynchronize(cs);
        for (int i = 0; i < 2; ++i) d_.host_sendrecv(h_send_[i], nb, right, h_recv_[i], left);
        for (int i = 0; i < 2; ++i)
          cudaMemcpyAsync(nxt[i].data_ptr(), h_recv_[i], nb, cudaMemcpyHostToDevice, cs);
      }
      cur[0] = nxt[0];
      cur[1] = nxt[1];
    }
    return out;
  }

  const Args& a_;
  Dist& d_;
  const Meta& m_;
  torch::Tensor q_, k_, v_;
  double scale_;
  torch::Tensor status_, qtp_, kvtp_;
  std::vector<int64_t> kv_lens_;
  std::unique_ptr<mgfa::RingEngine> eng_;
  std::unique_ptr<mgfa::RingEngineP> peng_;
  torch::Tensor host_out_;    // pinned download target of the output
  torch::Tensor recv_[2][2];  // two receive pairs (K, V)
  void* h_send_[2] = {nullptr, nullptr};
  void* h_recv_[2] = {nullptr, nullptr};
  c10::cuda::CUDAStream comm_ = c10::cuda::getDefaultCUDAStream();
};

template <class T>
std::string json_list(const std::vector<T>& v) {
  std::string s = "[";
  for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(v[i]);
  return s + "]";
}

// The kernels' tables for every rank of a `world`-rank ring (one JSON line per
// rank), without touching a GPU: the layout logic is checked against the Python
// layer on the host.
int print_tables(const Args& a) {
  const int P = a.print_tables, D = a.head_dim ? a.head_dim : 128;
  const int64_t L = a.kv_size / (int64_t(a.heads) * D * 4);
  const Meta m = make_meta(a, L * P, P);
  for (int r = 0; r < P; ++r) {
    std::string kv = "[", kpos = "[";
    for (int o = 0; o < P; ++o) {
      kv += (o ? ", " : "") + json_list(m.kv_tile_pos(r, o));
      kpos += (o ? ", " : "") + json_list(m.k_positions(r, o));
    }
    std::printf("{\"rank\": %d, \"L\": %lld, \"q_tile_pos\": %s, \"kv_tile_pos\": %s]"
                ", \"q_positions\": %s, \"k_positions\": %s], \"local_len\": %lld}\n",
                r, (long long)m.L, json_list(m.tile_starts(r)).c_str(), kv.c_str(),
                json_list(m.q_positions(r)).c_str(), kpos.c_str(),
                (long long)m.plan.local_len(r));
  }
  return 0;
}

}  // namespace

static int run_main(int argc, char** argv) {
  Args a;
  if (!parse(argc, argv, &a)) {
    std::printf("Usage: ring_attention_bench <kv_size_bytes> [warmup] [iters] "
                "[--backend fused|fused_stepwise|fused_one_launch|p2p_unfused|ce_unfused|nccl|staged|p2p|ce] "
                "[--numerics fp32|bf16] "
                "[--init legacy|randn] "
                "[--layout contiguous|zigzag|striped|scheduler] [--policy dp|lpt] [--causal] "
                "[--heads H] [--kv-heads H] [--head-dim D] [--seed S] [--overlap] [--json]\n");
    return 1;
  }
  if (a.print_tables > 0) return print_tables(a);
  Dist d = Dist::from_env();
  const int P = d.world(), r = d.rank();
  auto log0 = [&](const std::string& s) {
    if (r == 0) std::printf("%s\n", s.c_str());
  };
  if (P < 2) {
    std::printf("Need at least 2 processes. Got %d.\n", P);
    return 1;
  }
  const int D = a.head_dim ? a.head_dim : (a.numerics == "bf16" ? 128 : 64);
  const int H = a.heads, Hkv = a.kv_heads ? a.kv_heads : a.heads;
  const int64_t unit = int64_t(H) * D * 4;
  if (!a.have_size) {
    log0("Usage: ring_attention_bench <kv_size_bytes> [warmup>=0] [iters>0]\nkv_size_bytes must be "
         "a positive multiple of " + std::to_string(unit) + " bytes.");
    return 1;
  }
  if (a.kv_size <= 0 || a.kv_size % unit != 0 || a.warmup < 0 || a.iters <= 0) {
    log0("Invalid arguments: kv_size must be a positive multiple of " + std::to_string(unit) +
         ", warmup >= 0, iters > 0.");
    return 1;
  }
  const bool exchange = a.backend == "p2p" || a.backend == "ce";
  if ((a.numerics == "fp32" && (D != 64 || (a.backend != "nccl" && a.backend != "staged" &&
                                            !exchange))) ||
      (a.numerics == "bf16" && exchange) || (a.overlap && exchange)) {
    log0("fp32 numerics: head_dim 64, backends nccl, staged, p2p or ce (p2p and ce run in the "
         "sequential order only)");
    return 1;
  }
  if (a.numerics == "bf16" && D != 64 && D != 128) {
    log0("bf16 numerics: head_dim 64 or 128");
    return 1;
  }
  if (a.init == "legacy" &&
      (H != 1 || a.layout != "contiguous" || a.causal || a.numerics != "fp32")) {
    log0("--init legacy is the reference's fp32 single-head, contiguous, non-causal setup");
    return 1;
  }
  const int64_t L = a.kv_size / unit, seq = L * P;
  Meta meta = make_meta(a, seq, P);
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, d.device());
  std::printf("[Rank %d local_rank %d] GPU %d: %s (%.0f MB total)\n", r, d.local_rank(),
              d.device(), prop.name, prop.totalGlobalMem / 1e6);
  const bool print_shards = std::getenv("ATTENTION_PRINT_SHARDS") != nullptr;
  if (print_shards) {
    if (a.layout == "contiguous")
      std::printf("[Rank %d] Q tokens=[%lld,%lld) KV tokens=[%lld,%lld) global_Q=%lld "
                  "global_KV=%lld\n",
                  r, (long long)(r * L), (long long)((r + 1) * L), (long long)(r * L),
                  (long long)((r + 1) * L), (long long)seq, (long long)seq);
    else
      std::printf("[Rank %d] Q tokens=%s KV tokens=%s global_Q=%lld global_KV=%lld\n", r,
                  meta.plan.describe(r).c_str(), meta.plan.describe(r).c_str(), (long long)seq,
                  (long long)seq);
  }
  std::printf("[Rank %d] seq_q=%lld, seq_k=%lld, dim=%d, KV shard=%.1f KB\n", r, (long long)L,
              (long long)L, D, double(L) * H * D * 4 / 1024.0);
  std::fflush(stdout);

  // inputs
  const double scale = a.init == "legacy" ? 1.0 : 1.0 / std::sqrt(double(D));
  const auto dev = torch::Device(torch::kCUDA, d.device());
  torch::Tensor q, k, v;
  if (a.init == "legacy") {
    const int64_t n = L * D;
    auto qh = torch::empty({n}, torch::kFloat32), kvh = torch::empty({n}, torch::kFloat32);
    float* pq = qh.data_ptr<float>();
    float* pk = kvh.data_ptr<float>();
    for (int64_t i = 0; i < n; ++i) {
      pq[i] = mgfa::synth::legacy_q(r, i, D);
      pk[i] = mgfa::synth::legacy_kv(r, i);
    }
    q = qh.view({L, 1, D}).to(dev);
    k = kvh.view({L, 1, D}).to(dev);
    v = k;
  } else {
    const auto rows = meta.plan.positions(r);
    auto mk = [&](uint64_t stream, int heads) {
      auto t = randn_rows(a.seed, stream, rows, meta.L, int64_t(heads) * D)
                   .view({meta.L, heads, D})
                   .to(dev);
      return a.numerics == "bf16" ? t.to(torch::kBFloat16).unsqueeze(0).contiguous() : t;
    };
    q = mk(mgfa::synth::kQ, H);
    k = mk(mgfa::synth::kK, Hkv);
    v = mk(mgfa::synth::kV, Hkv);
  }

  std::unique_ptr<Fp32Ring> f32;
  std::unique_ptr<Bf16Ring> b16;
  if (a.numerics == "fp32") f32 = std::make_unique<Fp32Ring>(a, d, meta, q, k, v, scale);
  else b16 = std::make_unique<Bf16Ring>(a, d, meta, q, k, v, scale);

  double sums[5] = {0, 0, 0, 0, 0};
  torch::Tensor host;
  for (int it = 0; it < a.warmup + a.iters; ++it) {
    d.barrier();
    StepTimes st = f32 ? f32->run(print_shards && it == 0) : b16->run(print_shards && it == 0);
    host = st.host;
    const auto mx = d.max({st.total, st.comm, st.attn, st.merge, st.final});
    if (it >= a.warmup)
      for (int i = 0; i < 5; ++i) sums[i] += mx[size_t(i)];
  }
  if (b16) {
    const int s = b16->status().item<int>();
    if (s) {
      std::fprintf(stderr, "[Rank %d] kernel status 0x%x\n", r, unsigned(s));
      return 1;
    }
  }
  const std::string name = a.backend + (a.overlap ? "_overlap" : "");
  const char* comm_name = a.backend == "nccl"                              ? "NCCL"
                          : a.backend == "staged"                          ? "MPI"
                          : a.backend == "ce_unfused" || a.backend == "ce" ? "CE"
                                                                           : "P2P";
  if (r == 0) {
    const double n = a.iters;
    std::printf("%s bench: warmup=%d iters=%d\n", name.c_str(), a.warmup, a.iters);
    std::printf("avg_total=%.3f ms avg_%s=%.3f avg_attn=%.3f avg_merge=%.3f avg_final=%.3f\n",
                sums[0] / n, comm_name, sums[1] / n, sums[2] / n, sums[3] / n, sums[4] / n);
    if (a.json) {
      const double pairs = a.causal ? double(seq) * double(seq + 1) / 2 : double(seq) * seq;
      // ring time: comm + attention + merge, without the final normalisation /
      // download of the output
      const double flops = 4.0 * D * H * pairs, ring = (sums[1] + sums[2] + sums[3]) / n;
      // roofline: the slower of the per-GPU FLOPs at the measured sustained bf16
      // peak and the KV bytes each rank sends at 770 GB/s (bf16 only)
      const double kv_bytes = double(P - 1) * 2.0 * double(meta.L) * Hkv * D * 2.0;
      const double t_roof =
          std::max(flops / P / (sustained_peak_tflops() * 1e12), kv_bytes / 770e9) * 1e3;
      const std::string roof =
          a.numerics == "bf16" && ring > 0 ? std::to_string(t_roof / ring) : "null";
      std::printf("{\"backend\": \"%s\", \"numerics\": \"%s\", \"ranks\": %d, \"seq\": %lld, "
                  "\"heads\": %d, \"head_dim\": %d, \"causal\": %s, \"layout\": \"%s\", "
                  "\"avg_total_ms\": %.4f, \"ring_ms\": %.4f, \"avg_comm_ms\": %.4f, "
                  "\"avg_attn_ms\": %.4f, \"tflops_per_gpu\": %.2f, \"roofline_fraction\": %s}\n",
                  name.c_str(), a.numerics.c_str(), P, (long long)seq, H, D,
                  a.causal ? "true" : "false", a.layout.c_str(), sums[0] / n, ring, sums[1] / n,
                  sums[2] / n, flops / (ring * 1e-3) / 1e12 / P, roof.c_str());
    }
    std::fflush(stdout);
  }
  if (std::getenv("ATTENTION_DUMP_OUTPUT")) {
    const std::string fname = "ring_output_rank" + std::to_string(r) + ".bin";
    auto h = host.contiguous();
    FILE* fp = std::fopen(fname.c_str(), "wb");
    if (!fp) {
      std::fprintf(stderr, "[Rank %d] cannot write %s\n", r, fname.c_str());
      return 1;
    }
    std::fwrite(h.data_ptr<float>(), sizeof(float), size_t(h.numel()), fp);
    std::fclose(fp);
    std::printf("[Rank %d] output dumped to %s\n", r, fname.c_str());
  }
  d.barrier();
  return 0;
}

int main(int argc, char** argv) {
  try {
    return run_main(argc, argv);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ring_attention_bench: %s\n", e.what());
    return 1;
  }
}
