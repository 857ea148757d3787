#include "symmetric.hpp"

#include <cstring>
#include <stdexcept>

namespace mgfa::comm {

namespace {
void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int d) {
    cudaGetDevice(&prev);
    if (prev != d) check(cudaSetDevice(d), "cudaSetDevice");
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

SymmetricBuffer::SymmetricBuffer(size_t payload_bytes, int rank, int world, int device,
                                 size_t flag_bytes)
    : rank_(rank),
      world_(world),
      device_(device),
      payload_bytes_((payload_bytes + 4095) & ~size_t(4095)),
      flag_bytes_((flag_bytes + 4095) & ~size_t(4095)) {
  if (world <= 0 || rank < 0 || rank >= world) throw std::invalid_argument("bad rank/world");
  DeviceScope ds(device_);
  void* p = nullptr;
  check(cudaMalloc(&p, flag_bytes_ + payload_bytes_), "cudaMalloc(symmetric buffer)");
  local_ = static_cast<uint8_t*>(p);
  check(cudaMemset(local_, 0, flag_bytes_), "cudaMemset(flags)");
  check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  peers_.assign(world_, nullptr);
  peers_[rank_] = local_;
}

SymmetricBuffer::~SymmetricBuffer() {
  DeviceScope ds(device_);
  for (int r = 0; r < world_; ++r)
    if (r != rank_ && peers_[r]) cudaIpcCloseMemHandle(peers_[r]);
  if (local_) cudaFree(local_);
}

std::string SymmetricBuffer::ipc_handle() const {
  DeviceScope ds(device_);
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, local_), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void SymmetricBuffer::open_peers(const std::vector<std::string>& handles) {
  if (int(handles.size()) != world_) throw std::invalid_argument("need one handle per rank");
  DeviceScope ds(device_);
  for (int r = 0; r < world_; ++r) {
    if (r == rank_) continue;
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t))
      throw std::invalid_argument("malformed IPC handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    peers_[r] = static_cast<uint8_t*>(p);
  }
  connected_ = true;
}

void SymmetricBuffer::reset_flags(cudaStream_t stream) {
  DeviceScope ds(device_);
  check(cudaMemsetAsync(local_, 0, flag_bytes_, stream), "cudaMemsetAsync(flags)");
}

}  // namespace mgfa::comm
