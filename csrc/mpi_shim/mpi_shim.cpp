// Implementation of the MPI subset in mpi.h for the ranks of one node: a
// shared-memory mailbox carries point-to-point messages and the barrier, CUDA
// IPC carries device buffers, and a c10d TCPStore does the rendezvous, the
// broadcast and reduce, and payloads too large for a mailbox slot.
//
// Matching: message n of the triple (src, dst, tag) carries sequence number n.
// Both sides count, so receives match sends in posting order (MPI's
// non-overtaking rule for one sender, tag and communicator).
//
// Mailbox: for every ordered pair (src, dst) a ring of slots in a POSIX shared
// memory segment. The sender claims a free slot (state 0), fills it and
// publishes it (state 1, release store); the receiver finds the slot with its
// tag and sequence number (acquire load), consumes it and frees it (state 0),
// or, for a device message, marks it copied (state 2) for the sender to free.
// One thread per process drives the shim (MPI_THREAD_FUNNELED), so each slot
// has one writer per transition. Slot kinds, chosen by the sender:
//  * 'H': a host payload small enough for the slot, inline; the send completes
//    once posted.
//  * 'B': a larger host payload, moved in pieces (1 MB, MPI_SHIM_PIECE_BYTES)
//    through a staging segment of shared memory that the sender keeps per
//    destination (created on demand, grown when idle, at most two pieces).
//    Each piece's slot names the segment, the piece's place in it and in the
//    message; the receiver copies the piece out and marks the slot copied
//    (state 2), which frees that half of the segment for the piece after
//    next, so copy-in and copy-out overlap and a piece is copied out while it
//    is still in the caches (1 MB pieces ran 16 MB messages at 5.7 GB/s on a
//    host whose plain memcpy runs at 3.8 GB/s; 4 MB pieces at 3.3, one piece
//    at 2.3). The send completes when every piece has been copied out.
//  * 'S': the same when no staging segment can be had (no room in
//    /dev/shm): the payload goes into the store under the message's key.
//  * 'D' (device buffer; MPI_SHIM_CUDA_IPC=0 turns it off): a CUDA IPC handle
//    of the allocation with its buffer id, offset and length, and the handle
//    of an IPC event (one from a pool per send in flight) recorded on the
//    legacy default stream at the send. The receiver opens the handle once
//    per (sender, buffer id), orders a copy-engine copy after that event on
//    its own non-blocking stream, and marks the slot copied when the copy has
//    finished. The send completes when the sender sees the mark; only then may
//    it reuse the buffer or the event. The payload crosses NVLink directly.
//    Allocations that cannot be exported (memory pools) are staged as 'B'.
//
// Progress: every wait, test and barrier advances all pending requests of the
// process (post queued sends, match slots, start copies, poll their events,
// free acknowledged slots), so blocking calls in any order cannot deadlock on
// an acknowledgement. Every wait yields between polls and gives up after
// MPI_SHIM_TIMEOUT_S seconds (default 600) with an error. The broadcast,
// reduce, gather and scatter wait in the store without driving progress.
#include "mpi.h"
#include "mpi_shim_ext.hpp"

#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <random>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

namespace mgfa_mpi_shim {

constexpr int kSlots = 16;               // per ordered pair of ranks
constexpr size_t kSlotBytes = 1024;
constexpr size_t kSlotHeader = 24;
constexpr size_t kInline = kSlotBytes - kSlotHeader;
constexpr int kMaxWorld = 32;            // 16 MB of mailboxes at 32 ranks

struct Slot {
  std::atomic<uint32_t> state;  // 0 free, 1 posted, 2 copied (sender frees)
  uint32_t kind;
  int32_t tag;
  uint32_t len;
  uint64_t seq;
  uint8_t data[kInline];
};
static_assert(sizeof(Slot) == kSlotBytes, "slot layout");
static_assert(std::atomic<uint32_t>::is_always_lock_free, "address-free atomics");

}  // namespace mgfa_mpi_shim

using mgfa_mpi_shim::Slot;

struct mgfa_mpi_request {
  enum Kind { kRecv, kSend } kind = kRecv;
  // send: kQueued (no free slot yet) -> kPosted ('D': waiting for the copy) -> kDone
  // receive: kPosted (matching) -> kCopying ('D') -> kDone
  enum Phase { kQueued, kPosted, kCopying, kDone } phase = kPosted;
  void* buf = nullptr;
  size_t bytes = 0;
  int source = 0, tag = 0;       // for a send: the destination and tag
  uint64_t seq = 0;
  char slot_kind = 'H';
  std::vector<uint8_t> record;   // send: the slot contents still to post
  const void* send_buf = nullptr; // send 'B': the payload, read when posted
  int event = -1;                 // send 'D': the pool event recorded at the send
  Slot* slot = nullptr;          // the slot this request posted or consumed
  cudaEvent_t copy_done = nullptr;
  // 'B' (staged) messages: bytes posted (send) or copied out (receive) so far,
  // the piece size, and the pieces in flight by half of the staging segment
  size_t done_bytes = 0;
  size_t piece = 0;
  Slot* pieces[2] = {nullptr, nullptr};
};

namespace {

using Clock = std::chrono::steady_clock;

struct IpcRecord {  // contents of a 'D' slot
  cudaIpcMemHandle_t mem;
  cudaIpcEventHandle_t event;
  uint64_t buffer_id = 0, offset = 0, bytes = 0;
  uint64_t address = 0;  // the sender's pointer, used as is when sender == receiver
};

struct Export {  // a device allocation of this process, exported for IPC
  char* base = nullptr;
  cudaIpcMemHandle_t handle;
};

struct IpcEvent {
  cudaEvent_t event = nullptr;
  cudaIpcEventHandle_t handle;
};

struct BulkRecord {  // contents of a 'B' slot: one piece of a staged message
  char name[64];
  uint64_t segment_bytes = 0;
  uint64_t offset = 0;      // of the piece in the message
  uint64_t seg_offset = 0;  // of the piece in the segment
  uint64_t bytes = 0;       // of the piece
  uint64_t total = 0;       // of the message
};

struct Segment {  // a named shared-memory segment, mapped in this process
  std::string name;
  char* ptr = nullptr;
  size_t size = 0;
  bool busy = false;  // staging: a posted message still lives in it
};

using mgfa_mpi_shim::kInline;
using mgfa_mpi_shim::kMaxWorld;
using mgfa_mpi_shim::kSlots;
static_assert(sizeof(IpcRecord) <= kInline, "IPC record fits a slot");
static_assert(sizeof(BulkRecord) <= kInline, "bulk record fits a slot");

struct SegmentHeader {
  std::atomic<uint32_t> barrier_count;
  std::atomic<uint32_t> barrier_generation;
  uint8_t pad[56];
};

struct State {
  int rank = 0, world = 1;
  c10::intrusive_ptr<c10d::Store> store;
  std::string prefix;
  std::map<std::tuple<int, int>, uint64_t> sent, received;  // (peer, tag) -> count
  uint64_t coll = 0;
  Clock::time_point t0 = Clock::now();
  double timeout_s = 600.0;
  bool ipc = true;
  // shared-memory segment: header, then world * world mailboxes of kSlots
  void* seg = nullptr;
  size_t seg_bytes = 0;
  std::vector<int> next_slot;              // per destination: where the free-slot scan starts
  std::vector<mgfa_mpi_request*> pending;  // started and not yet complete
  std::vector<Segment> staging;            // per destination ('B' sends)
  std::vector<Segment> mapped;             // per source: its staging segment, mapped here
  uint64_t staging_serial = 0;
  size_t piece_bytes = size_t(1) << 20;    // 'B' piece size
  // device side, created on first use on the current device
  std::map<uint64_t, Export> exports;     // buffer id -> export
  std::vector<IpcEvent> events;           // pool; a send holds one until it completes
  std::vector<int> free_events;
  cudaStream_t copy_stream = nullptr;
  std::map<std::string, char*> opened_mem;            // "<src>/<buffer id>" -> mapped base
  std::map<std::string, cudaEvent_t> opened_events;   // handle bytes -> event
  bool warned_ipc = false;

  SegmentHeader* header() const { return static_cast<SegmentHeader*>(seg); }
  Slot* mailbox(int src, int dst) const {
    return reinterpret_cast<Slot*>(static_cast<char*>(seg) + sizeof(SegmentHeader)) +
           size_t(src * world + dst) * kSlots;
  }
};

State* g = nullptr;

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

size_t type_size(MPI_Datatype t) {
  switch (t) {
    case MPI_BYTE:
    case MPI_CHAR:
      return 1;
    case MPI_INT:
    case MPI_FLOAT:
      return 4;
    case MPI_DOUBLE:
      return 8;
    default:
      throw std::runtime_error("unsupported MPI datatype " + std::to_string(t));
  }
}

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

bool on_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // no device, or memory the runtime does not know: host
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

void read_into(void* host, const void* buf, size_t bytes) {
  if (bytes == 0) return;
  if (on_device(buf)) cuda_ok(cudaMemcpy(host, buf, bytes, cudaMemcpyDeviceToHost), "D2H");
  else std::memcpy(host, buf, bytes);
}

std::vector<uint8_t> read_buffer(const void* buf, size_t bytes) {
  std::vector<uint8_t> v(bytes);
  read_into(v.data(), buf, bytes);
  return v;
}

void write_buffer(void* buf, const uint8_t* src, size_t n, size_t capacity) {
  if (n > capacity) throw std::runtime_error("message longer than the receive buffer");
  if (n == 0) return;
  if (on_device(buf)) cuda_ok(cudaMemcpy(buf, src, n, cudaMemcpyHostToDevice), "H2D");
  else std::memcpy(buf, src, n);
}

std::string msg_key(int src, int dst, int tag, uint64_t n) {
  return g->prefix + "m/" + std::to_string(src) + "/" + std::to_string(dst) + "/" +
         std::to_string(tag) + "/" + std::to_string(n);
}

std::string coll_key(const char* kind) {
  return g->prefix + kind + "/" + std::to_string(g->coll++);
}

std::string bytes_of(const void* p, size_t n) {
  return std::string(static_cast<const char*>(p), n);
}

int fail(const char* where, const std::exception& e) {
  std::fprintf(stderr, "[mpi shim rank %d] %s: %s\n", g ? g->rank : -1, where, e.what());
  return MPI_ERR_OTHER;
}

// Bounded poll loop: `done()` is re-evaluated after driving progress.
template <class F>
void spin_until(F done, const char* what);

// ------------------------------------------------------------------ device sends
template <class Fn>
Fn driver_fn(const char* name) {
  cudaDriverEntryPointQueryResult q;
  void* f = nullptr;
  cuda_ok(cudaGetDriverEntryPointByVersion(name, &f, 12000, cudaEnableDefault, &q),
          "driver entry point");
  if (q != cudaDriverEntryPointSuccess || !f)
    throw std::runtime_error(std::string(name) + " unavailable");
  return reinterpret_cast<Fn>(f);
}

// The allocation holding p: its IPC export (cached per buffer id, which the
// driver makes unique per allocation in this process, so a freed and
// reallocated range is exported afresh).
const Export& export_allocation(const void* p, uint64_t* buffer_id) {
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  using AttrFn = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);
  static const RangeFn range = driver_fn<RangeFn>("cuMemGetAddressRange");
  static const AttrFn attr = driver_fn<AttrFn>("cuPointerGetAttribute");
  const CUdeviceptr dp = reinterpret_cast<CUdeviceptr>(p);
  unsigned long long id = 0;
  if (attr(&id, CU_POINTER_ATTRIBUTE_BUFFER_ID, dp) != CUDA_SUCCESS)
    throw std::runtime_error("no buffer id for a device pointer");
  *buffer_id = id;
  auto it = g->exports.find(id);
  if (it != g->exports.end()) return it->second;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, dp) != CUDA_SUCCESS) throw std::runtime_error("no allocation range");
  Export e;
  e.base = reinterpret_cast<char*>(base);
  cuda_ok(cudaIpcGetMemHandle(&e.handle, e.base), "memory handle");
  return g->exports.emplace(id, e).first->second;
}

// An interprocess event from the pool (one per send in flight).
int take_event() {
  if (g->free_events.empty()) {
    IpcEvent e;
    cuda_ok(cudaEventCreateWithFlags(&e.event, cudaEventDisableTiming | cudaEventInterprocess),
            "event create");
    cuda_ok(cudaIpcGetEventHandle(&e.handle, e.event), "event handle");
    g->events.push_back(e);
    g->free_events.push_back(int(g->events.size()) - 1);
  }
  const int i = g->free_events.back();
  g->free_events.pop_back();
  return i;
}

std::vector<uint8_t> device_record(const void* buf, size_t bytes, int* event) {
  IpcRecord r;
  const Export& e = export_allocation(buf, &r.buffer_id);
  r.mem = e.handle;
  r.offset = uint64_t(static_cast<const char*>(buf) - e.base);
  r.bytes = bytes;
  r.address = reinterpret_cast<uint64_t>(buf);
  *event = take_event();
  r.event = g->events[size_t(*event)].handle;
  // everything the program queued before the send (legacy stream semantics)
  cuda_ok(cudaEventRecord(g->events[size_t(*event)].event, cudaStreamLegacy), "event record");
  std::vector<uint8_t> v(sizeof(r));
  std::memcpy(v.data(), &r, sizeof(r));
  return v;
}

// ------------------------------------------------------------------ staging
void unmap(Segment& seg, bool unlink) {
  if (seg.ptr) munmap(seg.ptr, seg.size);
  if (unlink && !seg.name.empty()) shm_unlink(seg.name.c_str());
  seg = Segment{};
}

// A staging segment of at least `bytes` for sends to `dst`; false when
// /dev/shm has no room (the caller falls back to the store).
bool ensure_staging(int dst, size_t bytes) {
  Segment& seg = g->staging[size_t(dst)];
  if (seg.ptr && seg.size >= bytes) return true;
  unmap(seg, true);  // idle: the receiver has copied everything out of it
  const size_t size = (bytes + (1u << 20) - 1) & ~size_t((1u << 20) - 1);
  const std::string name = "/mgfa_mpi_" + std::to_string(getpid()) + "_" + std::to_string(dst) +
                           "_" + std::to_string(g->staging_serial++);
  const int fd = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0) return false;
  // reserve the pages now, so that a full /dev/shm is an error here rather
  // than a bus error on first touch
  void* p = MAP_FAILED;
  if (posix_fallocate(fd, 0, off_t(size)) == 0)
    p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    shm_unlink(name.c_str());
    return false;
  }
  seg.name = name;
  seg.ptr = static_cast<char*>(p);
  seg.size = size;
  return true;
}

const Segment& map_from(int src, const BulkRecord& r) {
  Segment& seg = g->mapped[size_t(src)];
  if (seg.ptr && seg.name == r.name) return seg;
  unmap(seg, false);  // the sender replaced it: it was idle
  const int fd = shm_open(r.name, O_RDWR, 0600);
  if (fd < 0) throw std::runtime_error(std::string("cannot open staging segment ") + r.name);
  void* p = mmap(nullptr, r.segment_bytes, PROT_READ, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) throw std::runtime_error("cannot map a staging segment");
  seg.name = r.name;
  seg.ptr = static_cast<char*>(p);
  seg.size = r.segment_bytes;
  return seg;
}

// ------------------------------------------------------------------ sends
// A free slot of the mailbox to `dst` (claimed for this process to fill), or null.
Slot* claim_slot(int dst) {
  Slot* box = g->mailbox(g->rank, dst);
  int& start = g->next_slot[size_t(dst)];
  for (int k = 0; k < kSlots; ++k) {
    Slot* c = box + (start + k) % kSlots;
    if (c->state.load(std::memory_order_acquire) == 0) {
      start = (start + k + 1) % kSlots;
      return c;
    }
  }
  return nullptr;
}

void publish(Slot* s, const mgfa_mpi_request* q, char kind, uint32_t len, const void* data,
             size_t n) {
  s->kind = uint32_t(kind);
  s->tag = q->tag;
  s->seq = q->seq;
  s->len = len;
  if (n) std::memcpy(s->data, data, n);
  s->state.store(1, std::memory_order_release);
}

// A started 'B' send: frees the halves whose pieces were copied out and posts
// the next pieces into free halves. True when every piece is posted and
// copied out.
bool pump_bulk(mgfa_mpi_request* q) {
  Segment& seg = g->staging[size_t(q->source)];
  for (Slot*& p : q->pieces) {
    if (p && p->state.load(std::memory_order_acquire) == 2) {
      p->state.store(0, std::memory_order_release);
      p = nullptr;
    }
  }
  while (q->done_bytes < q->bytes) {
    const int h = !q->pieces[0] ? 0 : !q->pieces[1] ? 1 : -1;
    if (h < 0) break;
    Slot* s = claim_slot(q->source);
    if (!s) break;
    const size_t n = std::min(q->piece, q->bytes - q->done_bytes);
    read_into(seg.ptr + size_t(h) * q->piece, static_cast<const char*>(q->send_buf) + q->done_bytes,
              n);
    BulkRecord r;
    std::snprintf(r.name, sizeof(r.name), "%s", seg.name.c_str());
    r.segment_bytes = seg.size;
    r.offset = q->done_bytes;
    r.seg_offset = size_t(h) * q->piece;
    r.bytes = n;
    r.total = q->bytes;
    publish(s, q, 'B', uint32_t(n), &r, sizeof(r));
    q->pieces[h] = s;
    q->done_bytes += n;
  }
  return q->done_bytes == q->bytes && !q->pieces[0] && !q->pieces[1];
}

// Starts a queued send: posts it into a free slot of the mailbox to its
// destination ('B': takes the destination's staging segment and posts the
// first pieces). False when it has to stay queued.
bool try_post(mgfa_mpi_request* q) {
  using R = mgfa_mpi_request;
  const int dst = q->source;
  if (q->slot_kind == 'B') {
    Segment& seg = g->staging[size_t(dst)];
    if (seg.busy) return false;  // another staged message to dst is under way
    q->piece = std::min(q->bytes, g->piece_bytes);
    const size_t halves = q->bytes > q->piece ? 2 : 1;
    if (ensure_staging(dst, halves * q->piece)) {
      seg.busy = true;
      q->phase = R::kPosted;
      pump_bulk(q);  // the first pieces, as far as slots are free
      return true;
    }
    q->slot_kind = 'S';  // no room in /dev/shm: the whole payload through the store
  }
  Slot* s = claim_slot(dst);
  if (!s) return false;
  if (q->slot_kind == 'S')
    g->store->set(msg_key(g->rank, dst, q->tag, q->seq), read_buffer(q->send_buf, q->bytes));
  const uint32_t len = uint32_t(q->slot_kind == 'H' ? q->record.size() : q->bytes);
  publish(s, q, q->slot_kind, len, q->record.data(), q->record.size());
  q->record.clear();
  q->slot = s;
  q->phase = q->slot_kind == 'D' ? R::kPosted : R::kDone;
  return true;
}

// ------------------------------------------------------------------ receives
void start_ipc_copy(mgfa_mpi_request* q, const IpcRecord& r) {
  if (r.bytes > q->bytes) throw std::runtime_error("message longer than the receive buffer");
  if (!g->copy_stream)
    cuda_ok(cudaStreamCreateWithFlags(&g->copy_stream, cudaStreamNonBlocking), "stream");
  const char* src = nullptr;
  cudaEvent_t ready = nullptr;
  if (q->source == g->rank) {  // a message to itself: this process's own buffer and event
    src = reinterpret_cast<const char*>(r.address);
    for (const IpcEvent& ev : g->events)
      if (std::memcmp(&ev.handle, &r.event, sizeof(r.event)) == 0) ready = ev.event;
    if (!ready) throw std::runtime_error("unknown event in a message to self");
  } else {
    const std::string mk = std::to_string(q->source) + "/" + std::to_string(r.buffer_id);
    auto m = g->opened_mem.find(mk);
    if (m == g->opened_mem.end()) {
      void* p = nullptr;
      cuda_ok(cudaIpcOpenMemHandle(&p, r.mem, cudaIpcMemLazyEnablePeerAccess), "open memory");
      m = g->opened_mem.emplace(mk, static_cast<char*>(p)).first;
    }
    src = m->second + r.offset;
    const std::string ek = bytes_of(&r.event, sizeof(r.event));
    auto e = g->opened_events.find(ek);
    if (e == g->opened_events.end()) {
      cudaEvent_t ev = nullptr;
      cuda_ok(cudaIpcOpenEventHandle(&ev, r.event), "open event");
      e = g->opened_events.emplace(ek, ev).first;
    }
    ready = e->second;
  }
  cuda_ok(cudaStreamWaitEvent(g->copy_stream, ready, 0), "stream wait");
  if (r.bytes)
    cuda_ok(cudaMemcpyAsync(q->buf, src, r.bytes, cudaMemcpyDefault, g->copy_stream),
            "peer copy");
  cuda_ok(cudaEventCreateWithFlags(&q->copy_done, cudaEventDisableTiming), "event create");
  cuda_ok(cudaEventRecord(q->copy_done, g->copy_stream), "event record");
  q->phase = mgfa_mpi_request::kCopying;
}

// The posted slot for receive q: its tag and sequence number and, for a
// staged message, the piece that starts where the copied part ends.
Slot* match(const mgfa_mpi_request* q) {
  Slot* box = g->mailbox(q->source, g->rank);
  for (int k = 0; k < kSlots; ++k) {
    Slot* s = box + k;
    if (s->state.load(std::memory_order_acquire) != 1 || s->tag != q->tag || s->seq != q->seq)
      continue;
    if (s->kind == 'B') {
      uint64_t off = 0;
      std::memcpy(&off, s->data + offsetof(BulkRecord, offset), sizeof(off));
      if (off != q->done_bytes) continue;
    }
    return s;
  }
  return nullptr;
}

// One step of progress on request q; returns true when it is complete.
bool advance(mgfa_mpi_request* q) {
  using R = mgfa_mpi_request;
  if (q->phase == R::kDone) return true;
  if (q->kind == R::kSend) {
    if (q->phase == R::kQueued && !try_post(q)) return false;
    if (q->phase == R::kDone) return true;
    if (q->slot_kind == 'B') {
      if (!pump_bulk(q)) return false;
      g->staging[size_t(q->source)].busy = false;
      q->phase = R::kDone;
      return true;
    }
    // 'D': the receiver marks the slot copied; this side frees it
    if (q->slot->state.load(std::memory_order_acquire) != 2) return false;
    q->slot->state.store(0, std::memory_order_release);
    if (q->event >= 0) g->free_events.push_back(q->event);
    q->event = -1;
    q->phase = R::kDone;
    return true;
  }
  if (q->phase == R::kPosted) {
    Slot* s = match(q);
    if (!s) return false;
    q->slot = s;
    if (s->kind == 'H') {
      write_buffer(q->buf, s->data, s->len, q->bytes);
      s->state.store(0, std::memory_order_release);
      q->phase = R::kDone;
      return true;
    }
    if (s->kind == 'S') {
      const std::string key = msg_key(q->source, g->rank, q->tag, q->seq);
      const std::vector<uint8_t> v = g->store->get(key);
      g->store->deleteKey(key);
      write_buffer(q->buf, v.data(), v.size(), q->bytes);
      s->state.store(0, std::memory_order_release);
      q->phase = R::kDone;
      return true;
    }
    if (s->kind == 'B') {  // the next piece (match() checks its offset)
      BulkRecord r;
      std::memcpy(&r, s->data, sizeof(r));
      if (r.total > q->bytes) throw std::runtime_error("message longer than the receive buffer");
      const Segment& seg = map_from(q->source, r);
      if (r.seg_offset + r.bytes > seg.size || r.offset + r.bytes > r.total)
        throw std::runtime_error("malformed staging record");
      write_buffer(static_cast<char*>(q->buf) + r.offset,
                   reinterpret_cast<const uint8_t*>(seg.ptr) + r.seg_offset, r.bytes,
                   q->bytes - r.offset);
      s->state.store(2, std::memory_order_release);
      q->done_bytes += r.bytes;
      if (q->done_bytes < r.total) return false;
      q->phase = R::kDone;
      return true;
    }
    if (s->kind != 'D') throw std::runtime_error("malformed mailbox slot");
    IpcRecord r;
    std::memcpy(&r, s->data, sizeof(r));
    start_ipc_copy(q, r);
  }
  const cudaError_t st = cudaEventQuery(q->copy_done);
  if (st == cudaErrorNotReady) return false;
  cuda_ok(st, "peer copy");
  cudaEventDestroy(q->copy_done);
  q->copy_done = nullptr;
  q->slot->state.store(2, std::memory_order_release);
  q->phase = R::kDone;
  return true;
}

// Advances every pending request once and drops the completed ones. After an
// error the remaining requests stay pending, untouched, and the error is
// rethrown.
void progress_all() {
  auto& p = g->pending;
  size_t keep = 0;
  std::exception_ptr err;
  for (size_t i = 0; i < p.size(); ++i) {
    bool done = false;
    if (!err) {
      try {
        done = advance(p[i]);
      } catch (...) {
        err = std::current_exception();
      }
    }
    if (!done) p[keep++] = p[i];
  }
  p.resize(keep);
  if (err) std::rethrow_exception(err);
}

template <class F>
void spin_until(F done, const char* what) {
  const auto t0 = Clock::now();
  for (int spins = 0;; ++spins) {
    progress_all();
    if (done()) return;
    if (std::chrono::duration<double>(Clock::now() - t0).count() > g->timeout_s)
      throw std::runtime_error(std::string("timed out waiting for ") + what);
    if (spins > 1024) std::this_thread::sleep_for(std::chrono::microseconds(20));
    else std::this_thread::yield();
  }
}

void fill_status(const mgfa_mpi_request* r, MPI_Status* st) {
  if (!st || !r) return;
  st->MPI_SOURCE = r->source;
  st->MPI_TAG = r->tag;
  st->MPI_ERROR = MPI_SUCCESS;
  st->count_bytes = int(r->bytes);
}

// ------------------------------------------------------------------ setup
void store_barrier(const char* name) {
  const std::string k = g->prefix + name;
  if (g->store->add(k, 1) == g->world) g->store->set(k + "/done", std::vector<uint8_t>{1});
  g->store->wait({k + "/done"});
}

void map_segment() {
  if (g->world > kMaxWorld)
    throw std::runtime_error("more than " + std::to_string(kMaxWorld) + " ranks");
  char host[256] = {0};
  gethostname(host, sizeof(host) - 1);
  g->store->set(g->prefix + "host/" + std::to_string(g->rank),
                std::vector<uint8_t>(host, host + std::strlen(host)));
  const std::vector<uint8_t> h0 = g->store->get(g->prefix + "host/0");
  if (std::string(h0.begin(), h0.end()) != host)
    throw std::runtime_error("this MPI subset runs the ranks of one node only");
  g->seg_bytes = sizeof(SegmentHeader) + size_t(g->world) * g->world * kSlots * sizeof(Slot);
  std::string name;
  int fd = -1;
  if (g->rank == 0) {
    std::random_device rd;
    name = "/mgfa_mpi_" + std::to_string(getpid()) + "_" + std::to_string(rd());
    fd = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
    // reserve the pages now (an error here, not a bus error on first touch)
    if (fd < 0 || posix_fallocate(fd, 0, off_t(g->seg_bytes)) != 0) {
      if (fd >= 0) {
        close(fd);
        shm_unlink(name.c_str());
      }
      throw std::runtime_error("cannot create the shared-memory segment " + name);
    }
    g->store->set(g->prefix + "shm", std::vector<uint8_t>(name.begin(), name.end()));
  } else {
    const std::vector<uint8_t> v = g->store->get(g->prefix + "shm");
    name.assign(v.begin(), v.end());
    fd = shm_open(name.c_str(), O_RDWR, 0600);
    if (fd < 0) throw std::runtime_error("cannot open the shared-memory segment " + name);
  }
  g->seg = mmap(nullptr, g->seg_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (g->seg == MAP_FAILED) {
    g->seg = nullptr;
    throw std::runtime_error("cannot map the shared-memory segment");
  }
  store_barrier("mapped");
  if (g->rank == 0) shm_unlink(name.c_str());  // lives on while mapped
  g->next_slot.assign(size_t(g->world), 0);
  g->staging.assign(size_t(g->world), Segment{});
  g->mapped.assign(size_t(g->world), Segment{});
}

}  // namespace

namespace {

State* new_state(int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) throw std::runtime_error("bad RANK / WORLD_SIZE");
  auto* s = new State();
  s->rank = rank;
  s->world = world;
  s->timeout_s = env_int("MPI_SHIM_TIMEOUT_S", 600);
  s->ipc = env_int("MPI_SHIM_CUDA_IPC", 1) != 0;
  if (const char* pb = std::getenv("MPI_SHIM_PIECE_BYTES"); pb && *pb)
    s->piece_bytes = std::max<size_t>(4096, std::strtoull(pb, nullptr, 10));
  const char* run = std::getenv("TORCHELASTIC_RUN_ID");
  s->prefix = std::string("mpi_shim/") + (run ? run : "") + "/";
  return s;
}

}  // namespace

void mgfa::mpi_shim::init_with_store(c10::intrusive_ptr<c10d::Store> store, int rank,
                                     int world, int timeout_s) {
  if (g) return;
  g = new_state(rank, world);
  if (timeout_s > 0) g->timeout_s = timeout_s;
  try {
    if (world > 1) {
      g->store = std::move(store);
      map_segment();
    }
  } catch (...) {
    delete g;
    g = nullptr;
    throw;
  }
}

extern "C" {

int MPI_Init_thread(int*, char***, int required, int* provided) {
  if (g) return MPI_SUCCESS;
  try {
    g = new_state(env_int("RANK", 0), env_int("WORLD_SIZE", 1));
    if (g->world > 1) {
      c10d::TCPStoreOptions o;
      o.port = uint16_t(env_int("MASTER_PORT", 29500));
      const char* agent = std::getenv("TORCHELASTIC_USE_AGENT_STORE");
      const bool use_agent = agent && std::string(agent) == "True";
      o.isServer = !use_agent && g->rank == 0;
      o.numWorkers = use_agent ? std::nullopt : std::optional<size_t>(size_t(g->world));
      o.waitWorkers = !use_agent;
      o.timeout = std::chrono::milliseconds(int64_t(g->timeout_s * 1000));
      const char* addr = std::getenv("MASTER_ADDR");
      g->store = c10::make_intrusive<c10d::TCPStore>(addr && *addr ? addr : "127.0.0.1", o);
      map_segment();
    }
    if (provided) *provided = required;
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    const int rc = fail("MPI_Init", e);
    delete g;
    g = nullptr;
    return rc;
  }
}

int MPI_Init(int* argc, char*** argv) {
  int provided = 0;
  return MPI_Init_thread(argc, argv, MPI_THREAD_SINGLE, &provided);
}

int MPI_Finalize(void) {
  if (!g) return MPI_SUCCESS;
  // every rank leaves together: no peer still reads this process's buffers,
  // event or mailbox, and the store's host (rank 0) outlives the others
  int rc = MPI_Barrier(MPI_COMM_WORLD);
  if (g->world > 1) {
    try {
      store_barrier("finalize");
    } catch (const std::exception& e) {
      rc = fail("MPI_Finalize", e);
    }
  }
  for (auto& m : g->opened_mem) cudaIpcCloseMemHandle(m.second);
  for (auto& e : g->opened_events) cudaEventDestroy(e.second);
  for (auto& e : g->events) cudaEventDestroy(e.event);
  if (g->copy_stream) cudaStreamDestroy(g->copy_stream);
  for (auto& m : g->mapped) unmap(m, false);
  for (auto& st : g->staging) unmap(st, true);  // every receiver is past the barrier
  if (g->seg) munmap(g->seg, g->seg_bytes);
  delete g;
  g = nullptr;
  return rc;
}

int MPI_Abort(MPI_Comm, int errorcode) {
  std::fprintf(stderr, "[mpi shim rank %d] MPI_Abort(%d)\n", g ? g->rank : -1, errorcode);
  std::fflush(stderr);
  std::exit(errorcode == 0 ? 1 : errorcode);
}

int MPI_Comm_rank(MPI_Comm, int* rank) {
  *rank = g ? g->rank : 0;
  return MPI_SUCCESS;
}

int MPI_Comm_size(MPI_Comm, int* size) {
  *size = g ? g->world : 1;
  return MPI_SUCCESS;
}

// One node: the shared-memory split of the world is the world itself.
int MPI_Comm_split_type(MPI_Comm comm, int, int, MPI_Info, MPI_Comm* newcomm) {
  *newcomm = comm;
  return MPI_SUCCESS;
}

int MPI_Comm_free(MPI_Comm* comm) {
  *comm = MPI_COMM_NULL;
  return MPI_SUCCESS;
}

double MPI_Wtime(void) {
  const auto now = Clock::now();
  return std::chrono::duration<double>(now - (g ? g->t0 : now)).count();
}

// Sense-reversing counter barrier in the segment; drives progress while waiting.
int MPI_Barrier(MPI_Comm) {
  if (!g || g->world == 1) return MPI_SUCCESS;
  try {
    SegmentHeader* h = g->header();
    const uint32_t gen = h->barrier_generation.load(std::memory_order_acquire);
    if (h->barrier_count.fetch_add(1, std::memory_order_acq_rel) == uint32_t(g->world - 1)) {
      h->barrier_count.store(0, std::memory_order_relaxed);
      h->barrier_generation.fetch_add(1, std::memory_order_release);
    } else {
      spin_until([&] { return h->barrier_generation.load(std::memory_order_acquire) != gen; },
                 "the barrier");
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Barrier", e);
  }
}

int MPI_Bcast(void* buffer, int count, MPI_Datatype datatype, int root, MPI_Comm) {
  if (!g || g->world == 1) return MPI_SUCCESS;
  try {
    const size_t bytes = size_t(count) * type_size(datatype);
    const std::string k = coll_key("bcast");
    if (g->rank == root) {
      g->store->set(k, read_buffer(buffer, bytes));
    } else {
      const std::vector<uint8_t> v = g->store->get(k);
      write_buffer(buffer, v.data(), v.size(), bytes);
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Bcast", e);
  }
}

int MPI_Reduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype, MPI_Op op,
               int root, MPI_Comm) {
  try {
    const size_t bytes = size_t(count) * type_size(datatype);
    std::vector<uint8_t> mine = read_buffer(sendbuf, bytes);
    if (!g || g->world == 1) {
      if (recvbuf != sendbuf) write_buffer(recvbuf, mine.data(), bytes, bytes);
      return MPI_SUCCESS;
    }
    const std::string k = coll_key("reduce");
    g->store->set(k + "/" + std::to_string(g->rank), mine);
    if (g->rank != root) return MPI_SUCCESS;
    auto fold = [&](auto* acc, const auto* x) {
      for (int i = 0; i < count; ++i) {
        if (op == MPI_MAX) acc[i] = x[i] > acc[i] ? x[i] : acc[i];
        else if (op == MPI_MIN) acc[i] = x[i] < acc[i] ? x[i] : acc[i];
        else if (op == MPI_SUM) acc[i] += x[i];
        else throw std::runtime_error("unsupported MPI_Op");
      }
    };
    std::vector<uint8_t> acc = g->store->get(k + "/0");
    for (int r = 1; r < g->world; ++r) {
      const std::vector<uint8_t> x = g->store->get(k + "/" + std::to_string(r));
      if (datatype == MPI_DOUBLE)
        fold(reinterpret_cast<double*>(acc.data()), reinterpret_cast<const double*>(x.data()));
      else if (datatype == MPI_FLOAT)
        fold(reinterpret_cast<float*>(acc.data()), reinterpret_cast<const float*>(x.data()));
      else if (datatype == MPI_INT)
        fold(reinterpret_cast<int*>(acc.data()), reinterpret_cast<const int*>(x.data()));
      else
        throw std::runtime_error("unsupported MPI_Reduce datatype");
    }
    for (int r = 0; r < g->world; ++r) g->store->deleteKey(k + "/" + std::to_string(r));
    write_buffer(recvbuf, acc.data(), bytes, bytes);
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Reduce", e);
  }
}

int MPI_Type_size(MPI_Datatype datatype, int* size) {
  try {
    *size = int(type_size(datatype));
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Type_size", e);
  }
}

int MPI_Get_count(const MPI_Status* status, MPI_Datatype datatype, int* count) {
  try {
    *count = status->count_bytes / int(type_size(datatype));
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Get_count", e);
  }
}

int MPI_Allreduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype,
                  MPI_Op op, MPI_Comm comm) {
  const int rc = MPI_Reduce(sendbuf, recvbuf, count, datatype, op, 0, comm);
  return rc != MPI_SUCCESS ? rc : MPI_Bcast(recvbuf, count, datatype, 0, comm);
}

// Gather, allgather and scatter go through the store: every rank's block under
// the call's key (host staging for device buffers, as the broadcast does).
int MPI_Gather(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
               int recvcount, MPI_Datatype recvtype, int root, MPI_Comm) {
  try {
    const size_t sb = size_t(sendcount) * type_size(sendtype);
    const size_t rb = size_t(recvcount) * type_size(recvtype);
    if (!g || g->world == 1) {
      if (g && g->rank == root) write_buffer(recvbuf, read_buffer(sendbuf, sb).data(), sb, rb);
      return MPI_SUCCESS;
    }
    const std::string k = coll_key("gather");
    g->store->set(k + "/" + std::to_string(g->rank), read_buffer(sendbuf, sb));
    if (g->rank != root) return MPI_SUCCESS;
    for (int r = 0; r < g->world; ++r) {
      const std::string kr = k + "/" + std::to_string(r);
      const std::vector<uint8_t> v = g->store->get(kr);
      g->store->deleteKey(kr);
      write_buffer(static_cast<char*>(recvbuf) + size_t(r) * rb, v.data(), v.size(), rb);
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Gather", e);
  }
}

int MPI_Allgather(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
                  int recvcount, MPI_Datatype recvtype, MPI_Comm comm) {
  try {
    const int rc = MPI_Gather(sendbuf, sendcount, sendtype, recvbuf, recvcount, recvtype, 0, comm);
    if (rc != MPI_SUCCESS) return rc;
    const int world = g ? g->world : 1;
    const size_t total = size_t(recvcount) * size_t(world);
    return MPI_Bcast(recvbuf, int(total), recvtype, 0, comm);
  } catch (const std::exception& e) {
    return fail("MPI_Allgather", e);
  }
}

int MPI_Scatter(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
                int recvcount, MPI_Datatype recvtype, int root, MPI_Comm) {
  try {
    const size_t sb = size_t(sendcount) * type_size(sendtype);
    const size_t rb = size_t(recvcount) * type_size(recvtype);
    if (!g || g->world == 1) {
      write_buffer(recvbuf, read_buffer(sendbuf, sb).data(), sb, rb);
      return MPI_SUCCESS;
    }
    const std::string k = coll_key("scatter");
    if (g->rank == root) {
      const std::vector<uint8_t> all = read_buffer(sendbuf, sb * size_t(g->world));
      for (int r = 0; r < g->world; ++r)
        g->store->set(k + "/" + std::to_string(r),
                      std::vector<uint8_t>(all.begin() + long(size_t(r) * sb),
                                           all.begin() + long(size_t(r + 1) * sb)));
    }
    const std::string mine = k + "/" + std::to_string(g->rank);
    const std::vector<uint8_t> v = g->store->get(mine);
    g->store->deleteKey(mine);
    write_buffer(recvbuf, v.data(), v.size(), rb);
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Scatter", e);
  }
}

int MPI_Isend(const void* buf, int count, MPI_Datatype datatype, int dest, int tag, MPI_Comm,
              MPI_Request* request) {
  try {
    if (!g || g->world == 1 || dest < 0 || dest >= g->world)
      throw std::runtime_error("bad destination (point-to-point needs 2 or more ranks)");
    auto* r = new mgfa_mpi_request();
    r->kind = mgfa_mpi_request::kSend;
    r->bytes = size_t(count) * type_size(datatype);
    r->source = dest;
    r->tag = tag;
    r->seq = g->sent[{dest, tag}]++;
    r->slot_kind = r->bytes <= kInline ? 'H' : 'B';
    if (g->ipc && r->bytes && on_device(buf)) {
      try {
        r->record = device_record(buf, r->bytes, &r->event);
        r->slot_kind = 'D';
      } catch (const std::exception& e) {  // e.g. memory-pool allocations: stage instead
        cudaGetLastError();
        if (!g->warned_ipc)
          std::fprintf(stderr, "[mpi shim rank %d] no CUDA IPC for a device buffer (%s); "
                       "staging through host memory\n", g->rank, e.what());
        g->warned_ipc = true;
      }
    }
    if (r->slot_kind == 'H') r->record = read_buffer(buf, r->bytes);
    if (r->slot_kind == 'B') r->send_buf = buf;  // copied into the staging segment when posted
    r->phase = mgfa_mpi_request::kQueued;
    if (!try_post(r) || r->phase != mgfa_mpi_request::kDone) g->pending.push_back(r);
    *request = r;
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Isend", e);
  }
}

int MPI_Irecv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm,
              MPI_Request* request) {
  try {
    if (!g || g->world == 1 || source < 0 || source >= g->world)
      throw std::runtime_error("bad source");
    auto* r = new mgfa_mpi_request();
    r->kind = mgfa_mpi_request::kRecv;
    r->buf = buf;
    r->bytes = size_t(count) * type_size(datatype);
    r->source = source;
    r->tag = tag;
    r->seq = g->received[{source, tag}]++;
    g->pending.push_back(r);
    *request = r;
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Irecv", e);
  }
}

int MPI_Waitall(int count, MPI_Request reqs[], MPI_Status statuses[]) {
  try {
    spin_until(
        [&] {
          for (int i = 0; i < count; ++i)
            if (reqs[i] && reqs[i]->phase != mgfa_mpi_request::kDone) return false;
          return true;
        },
        "a message");
    for (int i = 0; i < count; ++i) {
      fill_status(reqs[i], statuses ? &statuses[i] : MPI_STATUS_IGNORE);
      delete reqs[i];
      reqs[i] = MPI_REQUEST_NULL;
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Waitall", e);
  }
}

int MPI_Wait(MPI_Request* request, MPI_Status* status) {
  return MPI_Waitall(1, request, status);
}

int MPI_Testall(int count, MPI_Request reqs[], int* flag, MPI_Status statuses[]) {
  try {
    progress_all();
    for (int i = 0; i < count; ++i) {
      if (reqs[i] && reqs[i]->phase != mgfa_mpi_request::kDone) {
        *flag = 0;
        return MPI_SUCCESS;
      }
    }
    *flag = 1;
    return MPI_Waitall(count, reqs, statuses);
  } catch (const std::exception& e) {
    return fail("MPI_Testall", e);
  }
}

int MPI_Send(const void* buf, int count, MPI_Datatype datatype, int dest, int tag,
             MPI_Comm comm) {
  MPI_Request r = MPI_REQUEST_NULL;
  const int rc = MPI_Isend(buf, count, datatype, dest, tag, comm, &r);
  return rc != MPI_SUCCESS ? rc : MPI_Wait(&r, MPI_STATUS_IGNORE);
}

int MPI_Recv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
             MPI_Status* status) {
  MPI_Request r = MPI_REQUEST_NULL;
  const int rc = MPI_Irecv(buf, count, datatype, source, tag, comm, &r);
  return rc != MPI_SUCCESS ? rc : MPI_Wait(&r, status);
}

// The receive is posted before the send, so two ranks exchanging device buffers
// with Sendrecv both make progress on their receive while waiting for the
// acknowledgement of their send.
int MPI_Sendrecv(const void* sendbuf, int sendcount, MPI_Datatype sendtype, int dest, int sendtag,
                 void* recvbuf, int recvcount, MPI_Datatype recvtype, int source, int recvtag,
                 MPI_Comm comm, MPI_Status* status) {
  MPI_Request r[2] = {MPI_REQUEST_NULL, MPI_REQUEST_NULL};
  int rc = MPI_Irecv(recvbuf, recvcount, recvtype, source, recvtag, comm, &r[0]);
  if (rc == MPI_SUCCESS) rc = MPI_Isend(sendbuf, sendcount, sendtype, dest, sendtag, comm, &r[1]);
  if (rc != MPI_SUCCESS) return rc;
  MPI_Status st[2];
  rc = MPI_Waitall(2, r, st);
  if (status) *status = st[0];
  return rc;
}

}  // extern "C"
