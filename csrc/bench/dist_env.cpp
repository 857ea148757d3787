#include "dist_env.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <thread>

#include "../common/device_select.hpp"
#include "../mpi_shim/mpi.h"
#include "../mpi_shim/mpi_shim_ext.hpp"

namespace mgfa::bench {

namespace {

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

std::vector<uint8_t> to_bytes(const void* p, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(p);
  return std::vector<uint8_t>(b, b + n);
}

}  // namespace

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess)
    throw std::runtime_error(std::string(what) + ": " + ncclGetErrorString(r));
}

Dist Dist::from_env(int timeout_s, bool need_gpu) {
  Dist d;
  d.timeout_s_ = timeout_s;
  d.world_ = env_int("WORLD_SIZE", 1);
  d.rank_ = env_int("RANK", 0);
  if (d.world_ < 1 || d.rank_ < 0 || d.rank_ >= d.world_)
    throw std::runtime_error("bad RANK / WORLD_SIZE");
  if (need_gpu) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
      throw std::runtime_error("no CUDA device");
    const auto choice = mgfa::choose_device(count, d.rank_);
    if (!choice.error.empty()) throw std::runtime_error(choice.error);
    d.local_rank_ = choice.local_rank;
    d.device_ = choice.device;
    if (cudaSetDevice(d.device_) != cudaSuccess) throw std::runtime_error("cudaSetDevice failed");
  } else {
    d.local_rank_ = mgfa::local_rank_from_env();
    d.device_ = -1;
  }
  if (d.world_ > 1) {
    const char* addr = std::getenv("MASTER_ADDR");
    c10d::TCPStoreOptions o;
    o.port = uint16_t(env_int("MASTER_PORT", 29500));
    const char* agent = std::getenv("TORCHELASTIC_USE_AGENT_STORE");
    const bool use_agent = agent && std::string(agent) == "True";
    o.isServer = !use_agent && d.rank_ == 0;
    o.numWorkers = use_agent ? std::nullopt : std::optional<size_t>(size_t(d.world_));
    o.waitWorkers = !use_agent;
    o.timeout = std::chrono::seconds(timeout_s);
    d.store_ = c10::make_intrusive<c10d::TCPStore>(addr && *addr ? addr : "127.0.0.1", o);
  }
  return d;
}

Dist& Dist::operator=(Dist&& o) noexcept {
  if (this != &o) {
    if (comm_) ncclCommDestroy(comm_);
    rank_ = o.rank_;
    world_ = o.world_;
    local_rank_ = o.local_rank_;
    device_ = o.device_;
    store_ = std::move(o.store_);
    coll_seq_ = o.coll_seq_;
    p2p_seq_ = o.p2p_seq_;
    comm_ = o.comm_;
    o.comm_ = nullptr;
    mpi_ = o.mpi_;
    o.mpi_ = false;
    store_p2p_ = o.store_p2p_;
    timeout_s_ = o.timeout_s_;
  }
  return *this;
}

Dist::~Dist() {
  if (comm_) ncclCommDestroy(comm_);
  if (mpi_) MPI_Finalize();  // collective, like every rank's destruction of its Dist
}

// Keys live under torchrun's run id (when set), so a reused agent store never
// hands a later run an earlier run's values.
std::string Dist::key(const char* kind, uint64_t seq) const {
  const char* run = std::getenv("TORCHELASTIC_RUN_ID");
  return std::string("mgfa_bench/") + (run ? run : "") + "/" + kind + "/" + std::to_string(seq);
}

void Dist::barrier() {
  if (world_ == 1) return;
  const std::string k = key("barrier", coll_seq_++);
  if (store_->add(k, 1) == world_) store_->set(k + "/done", {1});
  store_->wait({k + "/done"});
}

std::vector<std::string> Dist::all_gather(const std::string& mine) {
  if (world_ == 1) return {mine};
  const std::string k = key("gather", coll_seq_++);
  store_->set(k + "/" + std::to_string(rank_), to_bytes(mine.data(), mine.size()));
  std::vector<std::string> out(static_cast<size_t>(world_));
  for (int r = 0; r < world_; ++r) {
    const auto v = store_->get(k + "/" + std::to_string(r));
    out[size_t(r)].assign(v.begin(), v.end());
  }
  return out;
}

std::vector<double> Dist::max(const std::vector<double>& v) {
  const auto all = all_gather(std::string(reinterpret_cast<const char*>(v.data()),
                                          v.size() * sizeof(double)));
  std::vector<double> out = v;
  for (const auto& s : all) {
    if (s.size() != v.size() * sizeof(double)) throw std::runtime_error("max: size mismatch");
    const double* p = reinterpret_cast<const double*>(s.data());
    for (size_t i = 0; i < v.size(); ++i) out[i] = std::max(out[i], p[i]);
  }
  return out;
}

void Dist::host_sendrecv(const void* send, size_t n, int to, void* recv, int from) {
  if (world_ == 1) {
    if (send != recv) std::memcpy(recv, send, n);
    return;
  }
  if (!mpi_ && !store_p2p_) {  // collective: every rank's first host_sendrecv
    try {
      mgfa::mpi_shim::init_with_store(store_, rank_, world_, timeout_s_);
      mpi_ = true;
    } catch (const std::exception& e) {  // e.g. no /dev/shm: every rank falls back
      std::fprintf(stderr, "[rank %d] shared-memory transport unavailable (%s); host send/recv "
                   "through the store\n", rank_, e.what());
      store_p2p_ = true;
    }
  }
  if (store_p2p_) {
    const uint64_t seq = p2p_seq_++;
    const std::string out_key =
        key("p2p", seq) + "/" + std::to_string(rank_) + "->" + std::to_string(to);
    const std::string in_key =
        key("p2p", seq) + "/" + std::to_string(from) + "->" + std::to_string(rank_);
    store_->set(out_key, to_bytes(send, n));
    const auto v = store_->get(in_key);
    if (v.size() != n) throw std::runtime_error("host_sendrecv: size mismatch");
    std::memcpy(recv, v.data(), n);
    store_->deleteKey(in_key);
    return;
  }
  // MPI counts are int: at most 1 GiB per message
  constexpr size_t kMax = size_t(1) << 30;
  const char* s = static_cast<const char*>(send);
  char* r = static_cast<char*>(recv);
  size_t off = 0;
  do {
    const int c = int(std::min(kMax, n - off));
    if (MPI_Sendrecv(s + off, c, MPI_BYTE, to, 0, r + off, c, MPI_BYTE, from, 0, MPI_COMM_WORLD,
                     MPI_STATUS_IGNORE) != MPI_SUCCESS)
      throw std::runtime_error("host_sendrecv: MPI_Sendrecv failed");
    off += size_t(c);
  } while (off < n);
}

ncclComm_t Dist::nccl() {
  if (comm_) return comm_;
  ncclUniqueId id;
  const std::string k = key("nccl_id", coll_seq_++);
  if (rank_ == 0) {
    nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
    store_->set(k, to_bytes(&id, sizeof(id)));
  } else {
    const auto v = store_->get(k);
    if (v.size() != sizeof(id)) throw std::runtime_error("bad NCCL id");
    std::memcpy(&id, v.data(), sizeof(id));
  }
  nccl_check(ncclCommInitRank(&comm_, world_, id, rank_), "ncclCommInitRank");
  return comm_;
}

}  // namespace mgfa::bench
