// Allocation-free variant of the attention backward (see attn_bwd_noalloc.h).
// No counterpart in the reference prototype.
//
// The scratch that the regular entry point allocates per call (lse2, delta,
// status, causal tile positions) lives here in a file-scope device array. Host
// code never uses the array's name as a device pointer: in host code that name
// is only a stand-in for the symbol, so each device's real address is looked up
// with cudaGetSymbolAddress (on every call outside stream capture; a captured
// call reuses the last address found on its device).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "attn_bwd_noalloc.h"
#include "flash_bwd_sm100.cuh"

namespace mgfa {
cudaError_t flash_bwd_preprocess_raw(const void* o, const void* dout, int64_t o_sb, int64_t o_ss,
                                     int64_t do_sb, int64_t do_ss, const float* lse, int B, int S,
                                     int H, int s_pad, float* lse2, float* delta,
                                     cudaStream_t stream);
cudaError_t flash_bwd_kernels_raw(const CUtensorMap& mq, const CUtensorMap& mdo,
                                  const CUtensorMap& mk, const CUtensorMap& mv,
                                  const BwdParams& p, cudaStream_t stream);
}  // namespace mgfa

namespace {

constexpr size_t kScratchBytes = MGFA_BWD_NOALLOC_SCRATCH_BYTES;
constexpr size_t kStatusBytes = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// tile_pos[t] = 128 * t for the first n tiles of each of the two tables.
__global__ void fill_tile_positions(int* q_pos, int n_q, int* k_pos, int n_k) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_q) q_pos[i] = 128 * i;
  if (i < n_k) k_pos[i] = 128 * i;
}

void report(const char* what, cudaError_t e) {
  std::fprintf(stderr, "mgfa_attn_bwd_noalloc: %s: %s\n", what, cudaGetErrorString(e));
}

// Device address of the scratch array on the current device. Outside stream
// capture the address is looked up on every call (cheap), so a call after a
// device reset, which reloads the module, sees the new array; under capture
// the address of the last uncaptured call on this device is reused.
int scratch_for_current_device(bool capturing, unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    report("cudaGetDevice", e);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  if (dev < 0 || dev >= kMaxDevices) return MGFA_NOALLOC_BAD_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!capturing) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      report("cudaGetSymbolAddress", e);
      return MGFA_NOALLOC_CUDA_ERROR;
    }
    g_scratch_ptr[dev] = p;
  } else if (!g_scratch_ptr[dev]) {
    std::fprintf(stderr,
                 "mgfa_attn_bwd_noalloc: first call on device %d is under stream capture; "
                 "make one call on this device outside capture first\n",
                 dev);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
  return MGFA_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int mgfa_attn_bwd_noalloc(
    const void* dout, const void* q, const void* k, const void* v, const void* out,
    const float* lse, float* dq, float* dk, float* dv, int batch, int seqlen_q, int seqlen_k,
    int heads_q, int heads_kv, float softmax_scale, int causal, void* stream_ptr) {
  if (!dout || !q || !k || !v || !out || !lse || !dq || !dk || !dv) return MGFA_NOALLOC_BAD_ARGUMENT;
  if (batch <= 0 || seqlen_q <= 0 || seqlen_k <= 0 || heads_q <= 0 || heads_kv <= 0 ||
      heads_q % heads_kv != 0 || !(softmax_scale > 0.f))
    return MGFA_NOALLOC_BAD_ARGUMENT;
  for (const void* p : {dout, q, k, v, out, static_cast<const void*>(dq),
                        static_cast<const void*>(dk), static_cast<const void*>(dv)})
    if (!aligned16(p)) return MGFA_NOALLOC_BAD_ARGUMENT;

  const int n_q_tiles = (seqlen_q + 127) / 128, n_kv_tiles = (seqlen_k + 127) / 128;
  const int sq_pad = n_q_tiles * 128;
  const size_t pos_bytes = (size_t(n_q_tiles) + size_t(n_kv_tiles)) * sizeof(int);
  const size_t pos_region = (pos_bytes + 255) & ~size_t(255);
  const size_t vec_elems = size_t(batch) * size_t(heads_q) * size_t(sq_pad);
  const size_t vec_bytes = (vec_elems * sizeof(float) + 255) & ~size_t(255);
  const size_t need = kStatusBytes + pos_region + 2 * vec_bytes;
  if (need > kScratchBytes) {
    std::fprintf(stderr,
                 "mgfa_attn_bwd_noalloc: this problem needs %zu bytes of scratch but the static "
                 "array holds %zu (batch * heads_q * ceil(seqlen_q/128)*128 must stay below "
                 "about %zu)\n",
                 need, kScratchBytes, (kScratchBytes - kStatusBytes - pos_region) / 8);
    return MGFA_NOALLOC_TOO_LARGE;
  }

  // An error left pending by earlier, unrelated work belongs to its owner:
  // report it without clearing it. From here on every error is this call's.
  cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) {
    report("a CUDA error was already pending on entry (left in place)", pending);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t ce = cudaStreamIsCapturing(stream, &cap);
  if (ce != cudaSuccess) {
    cudaGetLastError();  // this call's own query error
    report("cudaStreamIsCapturing", ce);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  unsigned char* scratch = nullptr;
  int rc = scratch_for_current_device(cap != cudaStreamCaptureStatusNone, &scratch);
  if (rc != MGFA_NOALLOC_OK) return rc;
  uint32_t* status = reinterpret_cast<uint32_t*>(scratch);
  int* q_pos = reinterpret_cast<int*>(scratch + kStatusBytes);
  int* k_pos = q_pos + n_q_tiles;
  float* lse2 = reinterpret_cast<float*>(scratch + kStatusBytes + pos_region);
  float* delta = reinterpret_cast<float*>(scratch + kStatusBytes + pos_region + vec_bytes);

  try {
    cudaError_t e = cudaMemsetAsync(status, 0, kStatusBytes, stream);  // the status starts at 0
    if (e != cudaSuccess) {
      report("cudaMemsetAsync", e);
      return MGFA_NOALLOC_CUDA_ERROR;
    }
    if (causal) {
      const int n = n_q_tiles > n_kv_tiles ? n_q_tiles : n_kv_tiles;
      fill_tile_positions<<<(n + 255) / 256, 256, 0, stream>>>(q_pos, n_q_tiles, k_pos, n_kv_tiles);
      if ((e = cudaGetLastError()) != cudaSuccess) {
        report("tile positions", e);
        return MGFA_NOALLOC_CUDA_ERROR;
      }
    }
    const int64_t q_ss = int64_t(heads_q) * 128, q_sb = q_ss * seqlen_q;
    const int64_t k_ss = int64_t(heads_kv) * 128, k_sb = k_ss * seqlen_k;
    e = mgfa::flash_bwd_preprocess_raw(out, dout, q_sb, q_ss, q_sb, q_ss, lse, batch, seqlen_q,
                                       heads_q, sq_pad, lse2, delta, stream);
    if (e != cudaSuccess) {
      report("preprocess launch", e);
      return MGFA_NOALLOC_CUDA_ERROR;
    }
    const CUtensorMap mq = mgfa::make_bshd_map(q, batch, seqlen_q, heads_q, q_sb, q_ss, 128);
    const CUtensorMap mdo = mgfa::make_bshd_map(dout, batch, seqlen_q, heads_q, q_sb, q_ss, 128);
    const CUtensorMap mk = mgfa::make_bshd_map(k, batch, seqlen_k, heads_kv, k_sb, k_ss, 128);
    const CUtensorMap mv = mgfa::make_bshd_map(v, batch, seqlen_k, heads_kv, k_sb, k_ss, 128);
    mgfa::BwdParams p;
    p.batch = batch;
    p.hq = heads_q;
    p.hkv = heads_kv;
    p.sq = seqlen_q;
    p.sk = seqlen_k;
    p.n_q_tiles = n_q_tiles;
    p.n_kv_tiles = n_kv_tiles;
    p.sq_pad = sq_pad;
    p.scale = softmax_scale;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;
    p.causal = causal ? 1 : 0;
    p.q_tile_pos = causal ? q_pos : nullptr;
    p.kv_tile_pos = causal ? k_pos : nullptr;
    p.lse2 = lse2;
    p.delta = delta;
    p.dq = dq;
    p.dk = dk;
    p.dv = dv;
    p.dq_batch_stride = q_sb;
    p.dq_row_stride = q_ss;
    p.dkv_batch_stride = k_sb;
    p.dkv_row_stride = k_ss;
    p.accumulate = 0;
    p.status = status;
    e = mgfa::flash_bwd_kernels_raw(mq, mdo, mk, mv, p, stream);
    if (e != cudaSuccess) {
      report("backward launch", e);
      return MGFA_NOALLOC_CUDA_ERROR;
    }
  } catch (const std::exception& ex) {  // tensor-map encoding failures
    std::fprintf(stderr, "mgfa_attn_bwd_noalloc: %s\n", ex.what());
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  return MGFA_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) int mgfa_attn_bwd_noalloc_status(
    unsigned int* host_status, void* stream_ptr) {
  if (!host_status) return MGFA_NOALLOC_BAD_ARGUMENT;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    if (e != cudaSuccess) report("cudaGetDevice", e);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    scratch = g_scratch_ptr[dev];
  }
  if (!scratch) {
    std::fprintf(stderr, "mgfa_attn_bwd_noalloc_status: no call was made on device %d yet\n",
                 dev);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  // The status word sits at the start of the scratch array (the call clears it
  // before its kernels run, stream-ordered).
  e = cudaMemcpyAsync(host_status, scratch, sizeof(unsigned int), cudaMemcpyDeviceToHost,
                      static_cast<cudaStream_t>(stream_ptr));
  if (e != cudaSuccess) {
    report("status copy", e);
    return MGFA_NOALLOC_CUDA_ERROR;
  }
  return MGFA_NOALLOC_OK;
}
