// Symmetric device buffers: every rank allocates the same layout with
// cudaMalloc, exports a CUDA IPC handle, and maps every peer's buffer into its
// own address space, so kernels can store into (and signal) a neighbour's
// memory over NVLink. Handles travel through whatever bootstrap the caller has
// (torch.distributed from Python, a TCP store from the standalone benchmarks).
//
// Layout of one buffer:
//   [0, flag_bytes)          flag words (kFlagBytes by default, each named flag on
//                            its own 128-byte line)
//   [flag_bytes, ...)        payload (receive slots), 4 KB aligned
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mgfa::comm {

constexpr size_t kFlagBytes = 64 * 1024;
constexpr size_t kFlagStride = 128;  // bytes between flag words

// Flag word indices (slot s of a ring buffer uses kArrivals0 + s, kCredit0 + s,
// kDone0 + s; up to kMaxSlots slots).
constexpr int kMaxSlots = 4;
enum FlagIndex : int {
  kArrivals0 = 0,   // chunks of slot s received (written by the left neighbour)
  kCredit0 = 4,     // uses of the right neighbour's slot s it finished (written by it)
  kDone0 = 8,       // CTAs of this rank finished with slot s in the current step
  kTag0 = 12,       // owner tag of the data in slot s (written by the left neighbour)
  kStatus = 16,     // device error word of the last call
  kHomeArrivals = 20,  // backward: final dK/dV of this rank's shard arrived (CTA count)
  kHomeCredit = 21,    // backward: right neighbour's finished uses of its home buffer
};

class SymmetricBuffer {
 public:
  // flag_bytes: size of the flag area (rounded up to 4 KB).
  SymmetricBuffer(size_t payload_bytes, int rank, int world, int device,
                  size_t flag_bytes = kFlagBytes);
  ~SymmetricBuffer();
  SymmetricBuffer(const SymmetricBuffer&) = delete;
  SymmetricBuffer& operator=(const SymmetricBuffer&) = delete;

  // 64-byte cudaIpcMemHandle_t of the local allocation.
  std::string ipc_handle() const;
  // Map every peer's buffer; `handles[r]` is rank r's ipc_handle().
  void open_peers(const std::vector<std::string>& handles);

  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  size_t payload_bytes() const { return payload_bytes_; }
  bool connected() const { return connected_; }

  uint8_t* base(int r) const { return r == rank_ ? local_ : peers_.at(r); }
  uint8_t* payload(int r) const { return base(r) + flag_bytes_; }
  // Flag word `index` of rank r's packed uint32 flag array (no 128-byte spacing).
  uint32_t* word(int r, size_t index) const {
    return reinterpret_cast<uint32_t*>(base(r)) + index;
  }
  size_t flag_bytes() const { return flag_bytes_; }
  uint32_t* flag(int r, int index) const {
    return reinterpret_cast<uint32_t*>(base(r) + size_t(index) * kFlagStride);
  }
  // Zero the local flag words (call on every rank, then barrier, before use).
  void reset_flags(cudaStream_t stream);

 private:
  int rank_, world_, device_;
  size_t payload_bytes_;
  size_t flag_bytes_;
  uint8_t* local_ = nullptr;
  std::vector<uint8_t*> peers_;
  bool connected_ = false;
};

}  // namespace mgfa::comm
