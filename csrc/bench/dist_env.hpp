// Process-group plumbing of the native benchmark executables (no MPI, no Python).
//
// Rank, world size and the rendezvous address come from torchrun-style
// environment variables (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR, MASTER_PORT);
// `torchrun --no-python build/bin/<bench> ...` launches them. Rendezvous uses a
// c10d TCPStore: the launcher's store when it offers one
// (TORCHELASTIC_USE_AGENT_STORE), otherwise rank 0 hosts it. On top of the store:
// barriers, all-gather of small blobs, max-over-ranks reductions of timings (the
// reference's MPI_Reduce(MAX), ring/attention/bench/ring_attention_nccl_gpu_bench.cu:409-416),
// blocking host send/recv (the staged transport, through the MPI subset's
// shared-memory mailbox and staging segments, csrc/mpi_shim) and the NCCL communicator of
// the NCCL baselines (unique id published through the store, as the reference
// broadcasts it with MPI_Bcast, ring_attention_nccl_gpu_bench.cu:231-238).
#pragma once

#include <nccl.h>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace mgfa::bench {

class Dist {
 public:
  // Reads the environment, binds this process to its local GPU (same rules as
  // the Python layer: MPI/Slurm/PMI local-rank variables or LOCAL_RANK) and
  // connects to the store. Throws std::runtime_error on a bad environment.
  // need_gpu=false skips the device binding (host-only use of the store).
  static Dist from_env(int timeout_s = 300, bool need_gpu = true);

  // Movable, not copyable: the NCCL communicator has one owner.
  Dist(Dist&& o) noexcept { *this = std::move(o); }
  Dist& operator=(Dist&& o) noexcept;
  Dist(const Dist&) = delete;
  Dist& operator=(const Dist&) = delete;
  ~Dist();

  int rank() const { return rank_; }
  int world() const { return world_; }
  int local_rank() const { return local_rank_; }
  int device() const { return device_; }

  void barrier();
  std::vector<std::string> all_gather(const std::string& mine);
  std::vector<double> max(const std::vector<double>& v);
  // Blocking exchange: send `n` bytes to rank `to`, receive `n` bytes from `from`.
  void host_sendrecv(const void* send, size_t n, int to, void* recv, int from);
  // NCCL communicator over all ranks, created on first use (collective).
  ncclComm_t nccl();

 private:
  Dist() = default;
  std::string key(const char* kind, uint64_t seq) const;

  int rank_ = 0, world_ = 1, local_rank_ = 0, device_ = 0;
  c10::intrusive_ptr<c10d::TCPStore> store_;
  uint64_t coll_seq_ = 0, p2p_seq_ = 0;
  ncclComm_t comm_ = nullptr;
  bool mpi_ = false;        // the MPI subset was started on store_ (host_sendrecv)
  bool store_p2p_ = false;  // it could not start: host_sendrecv goes through the store
  int timeout_s_ = 300;     // bound of the store's and the MPI subset's waits
};

// Prints "[tag] NCCL error ..." and aborts the process group on failure.
void nccl_check(ncclResult_t r, const char* what);

}  // namespace mgfa::bench
