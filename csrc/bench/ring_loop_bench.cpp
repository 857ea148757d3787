// Native pure ring-exchange benchmark: the reference's ring/loop programs
// (ring_loop_{staged,staged_Isendrecv,cuda_aware,cuda_aware_Isendrecv,nccl}.cu)
// as one executable with a --backend flag, without MPI.
//
//   torchrun --nproc-per-node N --no-python build/bin/ring_loop_bench
//       <kv_size_bytes> [warmup=10] [iters=100] [--backend p2p|ce|nccl|staged]
//       [--payload-tokens T] [--kv-heads 8] [--ctas C] [--seed S] [--json]
//
// A kv_size_bytes buffer (float32 rank*1000 + i, ring_loop_nccl.cu:131-140)
// rotates around the ring for world-1 steps. One untimed pass first checks the
// first float received at step s against 1000 * ((rank - s - 1) mod P)
// (ring_loop_nccl.cu:146-176). Each timed iteration is bracketed by CUDA events
// on the launching stream, reduced with MAX over ranks; rank 0 prints the
// reference's RESULT line (ring_loop_nccl.cu:227-238) with payload
// (world-1) * kv_size. --payload-tokens T sends the bf16 K+V payload
// [T x kv_heads x 128 x 2] of seeded uniform values instead and checks whole
// buffers.
//
// Backends: p2p (all-SM push kernel over NVLink peer memory), ce (copy engine
// into the peer mapping + flag kernels), nccl (grouped ncclSend/ncclRecv per
// step), staged (device -> pinned host -> host send/recv through the store ->
// device).
#include <ATen/cuda/CUDAContext.h>
#include <cuda_runtime.h>
#include <torch/types.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../comm/ring_exchange.hpp"
#include "../common/synth.hpp"
#include "dist_env.hpp"

using mgfa::bench::Dist;

namespace {

struct Args {
  int64_t kv_size = 262144;
  int warmup = 10, iters = 100;
  std::string backend = "p2p";
  int64_t payload_tokens = 0;
  int kv_heads = 8;
  int ctas = 0;
  uint64_t seed = 0;
  bool json = false;
};

bool parse(int argc, char** argv, Args* a) {
  int pos = 0;
  for (int i = 1; i < argc; ++i) {
    std::string s = argv[i];
    auto next = [&]() -> const char* { return i + 1 < argc ? argv[++i] : nullptr; };
    if (s == "--backend") {
      const char* v = next();
      if (!v) return false;
      a->backend = v;
    } else if (s == "--payload-tokens") {
      const char* v = next();
      if (!v) return false;
      a->payload_tokens = std::atoll(v);
    } else if (s == "--kv-heads") {
      const char* v = next();
      if (!v) return false;
      a->kv_heads = std::atoi(v);
    } else if (s == "--ctas") {
      const char* v = next();
      if (!v) return false;
      a->ctas = std::atoi(v);
    } else if (s == "--seed") {
      const char* v = next();
      if (!v) return false;
      a->seed = uint64_t(std::atoll(v));
    } else if (s == "--json") {
      a->json = true;
    } else if (!s.empty() && s[0] == '-') {
      return false;
    } else {
      if (pos == 0) a->kv_size = std::atoll(s.c_str());
      else if (pos == 1) a->warmup = std::atoi(s.c_str());
      else if (pos == 2) a->iters = std::atoi(s.c_str());
      else return false;
      ++pos;
    }
  }
  return a->backend == "p2p" || a->backend == "ce" || a->backend == "nccl" ||
         a->backend == "staged";
}

// The buffer rank `owner` starts with (host copy).
std::vector<uint8_t> owner_data(const Args& a, int owner, int64_t nbytes) {
  std::vector<uint8_t> out(static_cast<size_t>(nbytes));
  if (a.payload_tokens) {
    const int64_t n = nbytes / 2;
    uint16_t* p = reinterpret_cast<uint16_t*>(out.data());
    const uint64_t stream = mgfa::synth::kPayload + 16 * uint64_t(owner);
    for (int64_t i = 0; i < n; ++i) {
      const float f = float(mgfa::synth::uniform(a.seed, stream, uint64_t(i)));
      uint32_t b;
      std::memcpy(&b, &f, 4);
      p[i] = uint16_t((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);  // round to nearest even
    }
  } else {
    float* p = reinterpret_cast<float*>(out.data());
    for (int64_t i = 0; i < nbytes / 4; ++i) p[i] = mgfa::synth::legacy_kv(owner, i);
  }
  return out;
}

#define CUDA_OK(x)                                                                    \
  do {                                                                                \
    cudaError_t e_ = (x);                                                             \
    if (e_ != cudaSuccess) {                                                          \
      std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, \
                   __LINE__);                                                         \
      std::exit(1);                                                                   \
    }                                                                                 \
  } while (0)

}  // namespace

static int run_main(int argc, char** argv) {
  Args a;
  if (!parse(argc, argv, &a)) {
    std::printf("Usage: ring_loop_bench <kv_size_bytes> [warmup] [iters] "
                "[--backend p2p|ce|nccl|staged] [--payload-tokens T] [--kv-heads H] "
                "[--ctas C] [--seed S] [--json]\n");
    return 1;
  }
  Dist d = Dist::from_env();
  const int P = d.world(), r = d.rank();
  if (P < 2) {
    std::printf("Need at least 2 processes. Got %d.\n", P);
    return 1;
  }
  const int64_t nbytes = a.payload_tokens ? a.payload_tokens * a.kv_heads * 128 * 2 * 2 : a.kv_size;
  if (nbytes <= 0 || nbytes % 32 != 0 || a.warmup < 0 || a.iters <= 0) {
    if (r == 0)
      std::printf("Invalid arguments: kv_size must be a positive multiple of 32, warmup >= 0, "
                  "iters > 0.\n");
    return 1;
  }
  const int right = (r + 1) % P, left = (r - 1 + P) % P;
  cudaDeviceProp prop;
  CUDA_OK(cudaGetDeviceProperties(&prop, d.device()));
  std::printf("[Rank %d] GPU %d: %s (%.0f MB total)\n", r, d.device(), prop.name,
              prop.totalGlobalMem / 1e6);
  std::printf("[Rank %d] KV shard: %lld bytes (%.1f KB), neighbors: left=%d right=%d\n", r,
              (long long)nbytes, nbytes / 1024.0, left, right);
  std::fflush(stdout);

  const auto init_h = owner_data(a, r, nbytes);
  const auto expect_last = owner_data(a, (r + 1) % P, nbytes);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto status = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, d.device()));
  const int64_t limit = 2000000000;

  // transport state
  std::unique_ptr<mgfa::RingExchange> ex;
  uint8_t *cur = nullptr, *nxt = nullptr, *h_send = nullptr, *h_recv = nullptr;
  uint8_t* bufs[2] = {nullptr, nullptr};
  int cur_i = 0;
  if (a.backend == "p2p" || a.backend == "ce") {
    const int n_ctas = a.ctas ? a.ctas : 2 * prop.multiProcessorCount;
    ex = std::make_unique<mgfa::RingExchange>(r, P, d.device(), (nbytes + 4095) / 4096 * 4096,
                                              n_ctas);
    ex->connect(d.all_gather(ex->ipc_handle()));
    CUDA_OK(cudaDeviceSynchronize());
    d.barrier();
  } else {
    CUDA_OK(cudaMalloc(&cur, size_t(nbytes)));
    CUDA_OK(cudaMalloc(&nxt, size_t(nbytes)));
    bufs[0] = cur;
    bufs[1] = nxt;
    if (a.backend == "staged") {
      CUDA_OK(cudaMallocHost(&h_send, size_t(nbytes)));
      CUDA_OK(cudaMallocHost(&h_recv, size_t(nbytes)));
    } else {
      d.nccl();
    }
  }
  auto reset = [&]() {
    if (ex) {
      CUDA_OK(cudaMemcpyAsync(ex->slot(0).data_ptr(), init_h.data(), size_t(nbytes),
                              cudaMemcpyHostToDevice, stream));
    } else {
      cur_i = 0;
      CUDA_OK(cudaMemcpyAsync(bufs[0], init_h.data(), size_t(nbytes), cudaMemcpyHostToDevice,
                              stream));
    }
    CUDA_OK(cudaStreamSynchronize(stream));
  };
  auto one_step = [&](int t) {
    if (ex) {
      ex->step(t, nbytes, a.backend, status, limit);
      return;
    }
    uint8_t* c = bufs[cur_i];
    uint8_t* n = bufs[cur_i ^ 1];
    if (a.backend == "nccl") {
      ncclComm_t comm = d.nccl();
      mgfa::bench::nccl_check(ncclGroupStart(), "ncclGroupStart");
      mgfa::bench::nccl_check(ncclSend(c, size_t(nbytes), ncclUint8, right, comm, stream), "ncclSend");
      mgfa::bench::nccl_check(ncclRecv(n, size_t(nbytes), ncclUint8, left, comm, stream), "ncclRecv");
      mgfa::bench::nccl_check(ncclGroupEnd(), "ncclGroupEnd");
      CUDA_OK(cudaStreamSynchronize(stream));
    } else {
      CUDA_OK(cudaMemcpyAsync(h_send, c, size_t(nbytes), cudaMemcpyDeviceToHost, stream));
      CUDA_OK(cudaStreamSynchronize(stream));
      d.host_sendrecv(h_send, size_t(nbytes), right, h_recv, left);
      CUDA_OK(cudaMemcpyAsync(n, h_recv, size_t(nbytes), cudaMemcpyHostToDevice, stream));
    }
    cur_i ^= 1;
  };
  auto received = [&](int t_last) -> const uint8_t* {
    return ex ? static_cast<const uint8_t*>(ex->slot((t_last + 1) & 1).data_ptr()) : bufs[cur_i];
  };
  auto release = [&]() {
    if (ex) ex->release(P - 1, a.backend, status, limit);
  };
  std::vector<uint8_t> host(static_cast<size_t>(nbytes));
  auto fetch = [&](const uint8_t* dev) {
    CUDA_OK(cudaStreamSynchronize(stream));
    CUDA_OK(cudaMemcpy(host.data(), dev, size_t(nbytes), cudaMemcpyDeviceToHost));
  };

  // untimed precheck
  reset();
  d.barrier();
  for (int t = 0; t < P - 1; ++t) {
    one_step(t);
    CUDA_OK(cudaStreamSynchronize(stream));
    d.barrier();
    const int owner = (r - t - 1 + P) % P;
    fetch(received(t));
    bool ok;
    if (a.payload_tokens) {
      ok = host == owner_data(a, owner, nbytes);
    } else {
      float first;
      std::memcpy(&first, host.data(), 4);
      ok = first == owner * 1000.0f;
    }
    if (!ok) {
      std::fprintf(stderr, "[Rank %d] %s precheck mismatch at step %d (expected owner %d)\n", r,
                   a.backend.c_str(), t, owner);
      return 1;
    }
  }
  release();
  CUDA_OK(cudaStreamSynchronize(stream));
  d.barrier();

  cudaEvent_t e0, e1;
  CUDA_OK(cudaEventCreate(&e0));
  CUDA_OK(cudaEventCreate(&e1));
  double sum_comm = 0, sum_total = 0;
  for (int rep = 0; rep < a.warmup + a.iters; ++rep) {
    reset();
    d.barrier();
    const auto w0 = std::chrono::steady_clock::now();
    CUDA_OK(cudaEventRecord(e0, stream));
    for (int t = 0; t < P - 1; ++t) one_step(t);
    release();
    CUDA_OK(cudaEventRecord(e1, stream));
    CUDA_OK(cudaEventSynchronize(e1));
    const double wall =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - w0).count();
    float ms = 0;
    CUDA_OK(cudaEventElapsedTime(&ms, e0, e1));
    const auto mx = d.max({double(ms), wall});
    if (rep >= a.warmup) {
      sum_comm += mx[0];
      sum_total += mx[1];
    }
  }
  if (status.item<int>() != 0) {
    std::fprintf(stderr, "[Rank %d] transport status 0x%x\n", r, status.item<int>());
    return 1;
  }
  fetch(received(P - 2));
  if (host != expect_last) {
    std::fprintf(stderr, "[Rank %d] final buffer is not owner %d's data\n", r, (r + 1) % P);
    return 1;
  }
  if (r == 0) {
    const double avg_c = sum_comm / a.iters, avg_t = sum_total / a.iters;
    const double payload = double(P - 1) * double(nbytes);
    const char* b = a.backend.c_str();
    std::printf("RESULT backend=%s bytes=%lld ranks=%d warmup=%d iters=%d avg_%s_ms=%.3f "
                "avg_total_ms=%.3f total_GBps=%.3f %s_GBps=%.3f\n",
                b, (long long)nbytes, P, a.warmup, a.iters, b, avg_c, avg_t,
                payload / (avg_t / 1e3) / 1e9, b, payload / (avg_c / 1e3) / 1e9);
    if (a.json) {
      // per-direction GB/s against the measured 770 GB/s peer-copy bandwidth
      const double gbps = payload / (avg_c / 1e3) / 1e9;
      std::printf("{\"backend\": \"%s\", \"bytes\": %lld, \"ranks\": %d, \"avg_ms\": %.4f, "
                  "\"per_direction_GBps\": %.2f, \"link_fraction\": %.3f, "
                  "\"payload_tokens\": %lld}\n",
                  b, (long long)nbytes, P, avg_c, gbps, gbps / 770.0, (long long)a.payload_tokens);
    }
    std::fflush(stdout);
  }
  d.barrier();
  if (cur) cudaFree(cur);
  if (nxt) cudaFree(nxt);
  if (h_send) cudaFreeHost(h_send);
  if (h_recv) cudaFreeHost(h_recv);
  return 0;
}

int main(int argc, char** argv) {
  try {
    return run_main(argc, argv);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ring_loop_bench: %s\n", e.what());
    return 1;
  }
}
