// Native one-shot legacy ring attention: the reference's ring/attention/gpu
// programs (ring_attention_{staged,cuda_aware,nccl}_gpu.cu) and its CPU-compute
// rings (ring/attention/ring_attention_{staged,cuda_aware}.cu) as one executable.
//
//   torchrun --nproc-per-node N --no-python build/bin/ring_oneshot
//       [--attention gpu|cpu] [--backend staged|nccl|p2p] [--seq 1024] [--dim 64]
//       [--cpu] [--out-dir DIR]
//
// One pass, no warm-up, as the reference: rank r holds Q and K == V of tokens
// [r*seq, (r+1)*seq) from the reference's formulas (kv[i] = 1000 r + i,
// q[i] = (500 r + 0.01 (i mod dim)) * 0.001, no softmax scale;
// gpu/ring_attention_staged_gpu.cu:240-262). The shard moves around the ring
// P-1 times; every rank prints its per-step phase times in the reference's
// format (gpu/ring_attention_staged_gpu.cu:364-442) and always writes
// ring_output_rank<r>.bin (fp32 [seq, dim]), which `verify_full <dir> N
// seq*dim*4` checks.
//
//   --attention gpu  fp32 partial attention + merge kernels (legacy_fp32.cu);
//                    dim 64
//   --attention cpu  the C++ host attention (csrc/host/cpu_attention.cpp)
//   --backend staged D2H, host send/recv (the MPI subset), H2D
//             nccl   NCCL send/recv of the device buffer (the role of the
//                    reference's CUDA-aware MPI)
//             p2p    the RingExchange push kernel over NVLink peer memory
//   --cpu            host memory only (--attention cpu --backend staged); runs
//                    without a GPU
//
// Phases are timed with the host clock around synchronous phases, as the
// reference's MPI_Wtime timers are.
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/types.h>

#include <cfloat>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../comm/ring_exchange.hpp"
#include "../host/cpu_attention.hpp"
#include "dist_env.hpp"

namespace mgfa {
void legacy_partial(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos,
                    bool causal, torch::Tensor acc, torch::Tensor m, torch::Tensor l, bool merge);
void legacy_merge(torch::Tensor m_run, torch::Tensor l_run, torch::Tensor acc_run,
                  torch::Tensor m_new, torch::Tensor l_new, torch::Tensor acc_new);
void legacy_normalize(torch::Tensor acc, torch::Tensor l, torch::Tensor out,
                      c10::optional<torch::Tensor> lse, c10::optional<torch::Tensor> m);
}  // namespace mgfa

using mgfa::bench::Dist;

namespace {

constexpr int64_t kWaitNs = 2000000000;

struct Args {
  std::string attention = "gpu", backend = "staged", out_dir = ".";
  int seq = 128 * 8, dim = 64;
  bool cpu = false;
};

bool parse(int argc, char** argv, Args* a) {
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto val = [&](std::string* out) {
      if (i + 1 >= argc) return false;
      *out = argv[++i];
      return true;
    };
    std::string v;
    if (s == "--attention") { if (!val(&a->attention)) return false; }
    else if (s == "--backend") { if (!val(&a->backend)) return false; }
    else if (s == "--out-dir") { if (!val(&a->out_dir)) return false; }
    else if (s == "--seq") { if (!val(&v)) return false; a->seq = std::atoi(v.c_str()); }
    else if (s == "--dim") { if (!val(&v)) return false; a->dim = std::atoi(v.c_str()); }
    else if (s == "--cpu") a->cpu = true;
    else return false;
  }
  return (a->attention == "gpu" || a->attention == "cpu") &&
         (a->backend == "staged" || a->backend == "nccl" || a->backend == "p2p") && a->seq > 0 &&
         a->dim > 0;
}

double now_ms() {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void sync() { cudaDeviceSynchronize(); }

// Running softmax state of the host attention.
struct HostState {
  std::vector<float> m, l, acc, m_loc, l_loc, acc_loc;
  HostState(int seq, int dim)
      : m(size_t(seq), -FLT_MAX), l(size_t(seq), 0.f), acc(size_t(seq) * dim, 0.f),
        m_loc(size_t(seq)), l_loc(size_t(seq)), acc_loc(size_t(seq) * dim) {}
};

int run(const Args& a, Dist& d) {
  const int P = d.world(), r = d.rank(), seq = a.seq, dim = a.dim;
  const int right = (r + 1) % P, left = (r - 1 + P) % P;
  const bool host_only = a.cpu, host_attn = a.attention == "cpu";
  const size_t n = size_t(seq) * dim, kv_bytes = n * 4;
  if (!host_only) {
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, d.device());
    std::printf("[Rank %d] GPU %d: %s (%.0f MB total)\n", r, d.device(), prop.name,
                double(prop.totalGlobalMem) / 1e6);
  }
  std::printf("[Rank %d] seq_q=%d, seq_k=%d, dim=%d, KV shard=%.1f KB\n", r, seq, seq, dim,
              double(kv_bytes) / 1024.0);
  std::fflush(stdout);

  // the reference's deterministic inputs, in float arithmetic as there
  std::vector<float> q(n), kv(n);
  for (size_t i = 0; i < n; ++i) {
    kv[i] = float(r) * 1000.0f + float(i);
    q[i] = (float(r) * 500.0f + float(i % size_t(dim)) * 0.01f) * 0.001f;
  }
  HostState hs(seq, dim);
  std::vector<float> h_send(n), h_recv(n);  // host staging (pageable: --cpu; pinned below)
  float* pin_send = nullptr;
  float* pin_recv = nullptr;

  auto f32 = torch::TensorOptions().dtype(torch::kFloat32);
  torch::Tensor q_dev, bufs[2], m_run, l_run, acc_run, m_loc, l_loc, acc_loc;
  std::unique_ptr<mgfa::RingExchange> ex;
  torch::Tensor status;
  if (!host_only) {
    auto dev = f32.device(torch::kCUDA, d.device());
    cudaMallocHost(reinterpret_cast<void**>(&pin_send), kv_bytes);
    cudaMallocHost(reinterpret_cast<void**>(&pin_recv), kv_bytes);
    q_dev = torch::from_blob(q.data(), {seq, 1, dim}, f32).to(dev);
    m_run = torch::empty({1, seq}, dev);
    l_run = torch::empty({1, seq}, dev);
    acc_run = torch::empty({seq, 1, dim}, dev);
    m_loc = torch::empty({1, seq}, dev);
    l_loc = torch::empty({1, seq}, dev);
    acc_loc = torch::empty({seq, 1, dim}, dev);
    status = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(dev.device()));
    if (a.backend == "p2p") {
      cudaDeviceProp prop;
      cudaGetDeviceProperties(&prop, d.device());
      ex = std::make_unique<mgfa::RingExchange>(r, P, d.device(),
                                                int64_t((kv_bytes + 4095) / 4096 * 4096),
                                                2 * prop.multiProcessorCount);
      ex->connect(d.all_gather(ex->ipc_handle()));
      ex->slot(0).narrow(0, 0, int64_t(kv_bytes))
          .copy_(torch::from_blob(kv.data(), {int64_t(kv_bytes)}, torch::kUInt8));
    } else {
      bufs[0] = torch::from_blob(kv.data(), {seq, 1, dim}, f32).to(dev);
      bufs[1] = torch::empty({seq, 1, dim}, dev);
    }
    if (a.backend == "nccl") {  // connect the pair untimed, as the reference's init does
      auto w = torch::zeros({2}, dev);
      ncclComm_t c = d.nccl();
      mgfa::bench::nccl_check(ncclGroupStart(), "ncclGroupStart");
      mgfa::bench::nccl_check(ncclSend(w.data_ptr(), 1, ncclFloat, right, c, nullptr), "ncclSend");
      mgfa::bench::nccl_check(ncclRecv(w[1].data_ptr(), 1, ncclFloat, left, c, nullptr), "ncclRecv");
      mgfa::bench::nccl_check(ncclGroupEnd(), "ncclGroupEnd");
    }
    sync();
  }
  d.barrier();

  auto slot_view = [&](int i) {
    return ex->slot(i).narrow(0, 0, int64_t(kv_bytes)).view(torch::kFloat32).view({seq, 1, dim});
  };
  // partial attention on one shard merged into the running state: (attn ms, merge ms)
  auto attend = [&](const float* kv_host, const torch::Tensor& kv_dev, bool first) {
    double t0 = now_ms(), t1, t2;
    if (host_attn) {
      mgfa::host::cpu_attention_partial(q.data(), seq, kv_host, kv_host, seq, dim, 1.f,
                                        hs.acc_loc.data(), hs.m_loc.data(), hs.l_loc.data());
      t1 = now_ms();
      mgfa::host::cpu_merge_online_softmax(hs.m.data(), hs.l.data(), hs.acc.data(),
                                           hs.m_loc.data(), hs.l_loc.data(), hs.acc_loc.data(),
                                           seq, dim);
      t2 = now_ms();
    } else {
      mgfa::legacy_partial(q_dev, kv_dev, kv_dev, 1.0, c10::nullopt, c10::nullopt, false, acc_loc,
                           m_loc, l_loc, false);
      sync();
      t1 = now_ms();
      if (first) {
        m_run.copy_(m_loc);
        l_run.copy_(l_loc);
        acc_run.copy_(acc_loc);
      } else {
        mgfa::legacy_merge(m_run, l_run, acc_run, m_loc, l_loc, acc_loc);
      }
      sync();
      t2 = now_ms();
    }
    return std::pair<double, double>{t1 - t0, t2 - t1};
  };

  const double t_start = now_ms();
  std::vector<float> cur_host = kv;  // host-only ring: the shard this rank forwards next
  if (host_only || host_attn) attend(kv.data(), torch::Tensor(), true);
  else attend(nullptr, ex ? slot_view(0) : bufs[0], true);
  std::printf("[Rank %d] step 0: attention on own KV\n", r);
  int cur = 0;
  for (int step = 0; step < P - 1; ++step) {
    const int src = ((r - step - 1) % P + P) % P;
    std::vector<std::pair<std::string, double>> parts;
    const float* recv_host = nullptr;
    torch::Tensor recv_dev;
    double t1 = now_ms();
    if (host_only) {
      d.host_sendrecv(cur_host.data(), kv_bytes, right, h_recv.data(), left);
      parts.push_back({"MPI", now_ms() - t1});
      cur_host.swap(h_recv);
      recv_host = cur_host.data();
    } else if (a.backend == "staged") {
      cudaMemcpy(pin_send, bufs[cur].data_ptr(), kv_bytes, cudaMemcpyDeviceToHost);
      const double t2 = now_ms();
      d.host_sendrecv(pin_send, kv_bytes, right, pin_recv, left);
      const double t3 = now_ms();
      cudaMemcpy(bufs[cur ^ 1].data_ptr(), pin_recv, kv_bytes, cudaMemcpyHostToDevice);
      const double t4 = now_ms();
      parts = {{"D2H", t2 - t1}, {"MPI", t3 - t2}, {"H2D", t4 - t3}};
      recv_dev = bufs[cur ^ 1];
      recv_host = pin_recv;
    } else {
      if (a.backend == "nccl") {
        ncclComm_t c = d.nccl();
        mgfa::bench::nccl_check(ncclGroupStart(), "ncclGroupStart");
        mgfa::bench::nccl_check(
            ncclSend(bufs[cur].data_ptr(), kv_bytes, ncclUint8, right, c, nullptr), "ncclSend");
        mgfa::bench::nccl_check(
            ncclRecv(bufs[cur ^ 1].data_ptr(), kv_bytes, ncclUint8, left, c, nullptr), "ncclRecv");
        mgfa::bench::nccl_check(ncclGroupEnd(), "ncclGroupEnd");
        sync();
        recv_dev = bufs[cur ^ 1];
      } else {
        ex->step(step, int64_t(kv_bytes), "p2p", status, kWaitNs);
        // the left neighbour's push into our slot may still be in flight
        ex->wait_received(step, "p2p", status, kWaitNs);
        sync();
        recv_dev = slot_view((step + 1) & 1);
      }
      const double t2 = now_ms();
      parts.push_back({a.backend == "nccl" ? "NCCL" : "P2P", t2 - t1});
      if (host_attn) {  // the host attention needs the shard in host memory
        cudaMemcpy(pin_recv, recv_dev.data_ptr(), kv_bytes, cudaMemcpyDeviceToHost);
        parts.push_back({"D2H", now_ms() - t2});
        recv_host = pin_recv;
      }
    }
    const auto [attn_ms, merge_ms] = attend(recv_host, recv_dev, false);
    double total = attn_ms + merge_ms;
    std::string body;
    for (const auto& p : parts) {
      char b[64];
      std::snprintf(b, sizeof(b), "%s%s=%.3f", body.empty() ? "" : " ", p.first.c_str(), p.second);
      body += b;
      total += p.second;
    }
    std::printf("[Rank %d] step %d: KV from rank %d | %s attn=%.3f merge=%.3f total=%.3f ms\n", r,
                step + 1, src, body.c_str(), attn_ms, merge_ms, total);
    std::fflush(stdout);
    cur ^= 1;
  }
  if (ex) ex->release(P - 1, "p2p", status, kWaitNs);
  std::vector<float> out(n);
  if (host_attn) {
    mgfa::host::cpu_normalize(hs.acc.data(), hs.l.data(), seq, dim);
    out = hs.acc;
  } else {
    auto o = torch::empty_like(acc_run);
    mgfa::legacy_normalize(acc_run, l_run, o, c10::nullopt, c10::nullopt);
    std::memcpy(out.data(), o.cpu().data_ptr<float>(), n * 4);
  }
  if (!host_only) sync();
  d.barrier();
  std::printf("[Rank %d] ring attention done in %.3f ms\n", r, now_ms() - t_start);
  int st = 0;
  if (status.defined()) st = status.item<int>();
  if (pin_send) cudaFreeHost(pin_send);
  if (pin_recv) cudaFreeHost(pin_recv);
  if (st != 0) {
    std::fprintf(stderr, "[Rank %d] transport status 0x%x\n", r, unsigned(st));
    return 1;
  }
  const std::string fname = "ring_output_rank" + std::to_string(r) + ".bin";
  FILE* fp = std::fopen((a.out_dir + "/" + fname).c_str(), "wb");
  if (!fp || std::fwrite(out.data(), 4, n, fp) != n) {
    std::fprintf(stderr, "[Rank %d] failed to write %s\n", r, fname.c_str());
    if (fp) std::fclose(fp);
    return 1;
  }
  std::fclose(fp);
  std::printf("[Rank %d] output dumped to %s\n", r, fname.c_str());
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  if (!parse(argc, argv, &a)) {
    std::printf("Usage: %s [--attention gpu|cpu] [--backend staged|nccl|p2p] [--seq N] "
                "[--dim D] [--cpu] [--out-dir DIR]\n", argv[0]);
    return 1;
  }
  if (a.attention == "gpu" && a.dim != 64) {
    std::printf("--attention gpu runs the fp32 kernels with dim 64\n");
    return 1;
  }
  if (a.cpu && (a.attention != "cpu" || a.backend != "staged")) {
    std::printf("--cpu runs --attention cpu --backend staged\n");
    return 1;
  }
  try {
    Dist d = Dist::from_env(300, !a.cpu);
    if (d.world() < 2) {
      std::printf("Need at least 2 processes. Got %d.\n", d.world());
      return 1;
    }
    return run(a, d);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ring_oneshot: %s\n", e.what());
    return 1;
  }
}
