// Implementation of the MPI subset in mpi.h over a c10d TCPStore.
//
// Point-to-point: a message from `src` to `dst` with tag `tag` is the store key
// .../m/<src>/<dst>/<tag>/<n>, where n counts the messages of that (src, dst,
// tag) triple on both sides, so receives match sends in posting order (MPI's
// non-overtaking rule for one sender, tag and communicator). Sends are eager
// (the store buffers them), so MPI_Isend completes at once; MPI_Irecv reserves
// its key when posted and completes in MPI_Wait / MPI_Waitall / MPI_Testall.
// Buffers in device memory are copied through host memory (cudaMemcpy), the
// behaviour of a CUDA-aware MPI. Collectives (barrier, broadcast, reduce) use
// keys numbered per call. Rendezvous: torchrun's store when it offers one
// (TORCHELASTIC_USE_AGENT_STORE), otherwise rank 0 hosts it.
#include "mpi.h"

#include <cuda_runtime.h>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

struct mgfa_mpi_request {
  bool is_recv = false;
  bool done = false;
  void* buf = nullptr;
  size_t bytes = 0;
  int source = 0, tag = 0;
  std::string key;
};

namespace {

struct State {
  int rank = 0, world = 1;
  c10::intrusive_ptr<c10d::TCPStore> store;
  std::string prefix;
  std::map<std::tuple<int, int>, uint64_t> sent, received;  // (peer, tag) -> count
  uint64_t coll = 0;
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
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

bool on_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // host memory the runtime does not know
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

std::vector<uint8_t> read_buffer(const void* buf, size_t bytes) {
  std::vector<uint8_t> v(bytes);
  if (bytes == 0) return v;
  if (on_device(buf)) {
    if (cudaMemcpy(v.data(), buf, bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
      throw std::runtime_error("device to host copy failed");
  } else {
    std::memcpy(v.data(), buf, bytes);
  }
  return v;
}

void write_buffer(void* buf, const std::vector<uint8_t>& v, size_t bytes) {
  if (v.size() > bytes) throw std::runtime_error("message longer than the receive buffer");
  if (v.empty()) return;
  if (on_device(buf)) {
    if (cudaMemcpy(buf, v.data(), v.size(), cudaMemcpyHostToDevice) != cudaSuccess)
      throw std::runtime_error("host to device copy failed");
  } else {
    std::memcpy(buf, v.data(), v.size());
  }
}

std::string msg_key(int src, int dst, int tag, uint64_t n) {
  return g->prefix + "m/" + std::to_string(src) + "/" + std::to_string(dst) + "/" +
         std::to_string(tag) + "/" + std::to_string(n);
}

std::string coll_key(const char* kind) {
  return g->prefix + kind + "/" + std::to_string(g->coll++);
}

int fail(const char* where, const std::exception& e) {
  std::fprintf(stderr, "[mpi shim rank %d] %s: %s\n", g ? g->rank : -1, where, e.what());
  return MPI_ERR_OTHER;
}

void complete_recv(mgfa_mpi_request* r, MPI_Status* st) {
  if (!r->done) {
    const std::vector<uint8_t> v = g->store->get(r->key);
    write_buffer(r->buf, v, r->bytes);
    g->store->deleteKey(r->key);
    r->done = true;
  }
  if (st) {
    st->MPI_SOURCE = r->source;
    st->MPI_TAG = r->tag;
    st->MPI_ERROR = MPI_SUCCESS;
    st->count_bytes = int(r->bytes);
  }
}

}  // namespace

extern "C" {

int MPI_Init_thread(int*, char***, int required, int* provided) {
  if (g) return MPI_SUCCESS;
  try {
    g = new State();
    g->world = env_int("WORLD_SIZE", 1);
    g->rank = env_int("RANK", 0);
    if (g->world < 1 || g->rank < 0 || g->rank >= g->world)
      throw std::runtime_error("bad RANK / WORLD_SIZE");
    const char* run = std::getenv("TORCHELASTIC_RUN_ID");
    g->prefix = std::string("mpi_shim/") + (run ? run : "") + "/";
    if (g->world > 1) {
      c10d::TCPStoreOptions o;
      o.port = uint16_t(env_int("MASTER_PORT", 29500));
      const char* agent = std::getenv("TORCHELASTIC_USE_AGENT_STORE");
      const bool use_agent = agent && std::string(agent) == "True";
      o.isServer = !use_agent && g->rank == 0;
      o.numWorkers = use_agent ? std::nullopt : std::optional<size_t>(size_t(g->world));
      o.waitWorkers = !use_agent;
      o.timeout = std::chrono::seconds(env_int("MPI_SHIM_TIMEOUT_S", 600));
      const char* addr = std::getenv("MASTER_ADDR");
      g->store = c10::make_intrusive<c10d::TCPStore>(addr && *addr ? addr : "127.0.0.1", o);
    }
    if (provided) *provided = required;
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Init", e);
  }
}

int MPI_Init(int* argc, char*** argv) {
  int provided = 0;
  return MPI_Init_thread(argc, argv, MPI_THREAD_SINGLE, &provided);
}

int MPI_Finalize(void) {
  if (!g) return MPI_SUCCESS;
  // every rank leaves together, so the store's host (rank 0) outlives the others
  MPI_Barrier(MPI_COMM_WORLD);
  delete g;
  g = nullptr;
  return MPI_SUCCESS;
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
  const auto now = std::chrono::steady_clock::now();
  const auto t0 = g ? g->t0 : now;
  return std::chrono::duration<double>(now - t0).count();
}

int MPI_Barrier(MPI_Comm) {
  if (!g || g->world == 1) return MPI_SUCCESS;
  try {
    const std::string k = coll_key("barrier");
    if (g->store->add(k, 1) == g->world) g->store->set(k + "/done", {1});
    g->store->wait({k + "/done"});
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
    if (g->rank == root) g->store->set(k, read_buffer(buffer, bytes));
    else write_buffer(buffer, g->store->get(k), bytes);
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
      if (recvbuf != sendbuf) write_buffer(recvbuf, mine, bytes);
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
    write_buffer(recvbuf, acc, bytes);
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Reduce", e);
  }
}

int MPI_Isend(const void* buf, int count, MPI_Datatype datatype, int dest, int tag, MPI_Comm,
              MPI_Request* request) {
  try {
    const size_t bytes = size_t(count) * type_size(datatype);
    const uint64_t n = g->sent[{dest, tag}]++;
    g->store->set(msg_key(g->rank, dest, tag, n), read_buffer(buf, bytes));
    if (request) {
      auto* r = new mgfa_mpi_request();
      r->done = true;
      *request = r;
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Isend", e);
  }
}

int MPI_Irecv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm,
              MPI_Request* request) {
  try {
    auto* r = new mgfa_mpi_request();
    r->is_recv = true;
    r->buf = buf;
    r->bytes = size_t(count) * type_size(datatype);
    r->source = source;
    r->tag = tag;
    r->key = msg_key(source, g->rank, tag, g->received[{source, tag}]++);
    *request = r;
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Irecv", e);
  }
}

int MPI_Wait(MPI_Request* request, MPI_Status* status) {
  try {
    if (*request) {
      if ((*request)->is_recv) complete_recv(*request, status);
      delete *request;
      *request = MPI_REQUEST_NULL;
    }
    return MPI_SUCCESS;
  } catch (const std::exception& e) {
    return fail("MPI_Wait", e);
  }
}

int MPI_Waitall(int count, MPI_Request reqs[], MPI_Status statuses[]) {
  for (int i = 0; i < count; ++i) {
    const int rc = MPI_Wait(&reqs[i], statuses ? &statuses[i] : MPI_STATUS_IGNORE);
    if (rc != MPI_SUCCESS) return rc;
  }
  return MPI_SUCCESS;
}

int MPI_Testall(int count, MPI_Request reqs[], int* flag, MPI_Status statuses[]) {
  try {
    for (int i = 0; i < count; ++i) {
      mgfa_mpi_request* r = reqs[i];
      if (r && r->is_recv && !r->done && !g->store->check({r->key})) {
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
  return MPI_Isend(buf, count, datatype, dest, tag, comm, nullptr);
}

int MPI_Recv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
             MPI_Status* status) {
  MPI_Request r = MPI_REQUEST_NULL;
  const int rc = MPI_Irecv(buf, count, datatype, source, tag, comm, &r);
  return rc != MPI_SUCCESS ? rc : MPI_Wait(&r, status);
}

int MPI_Sendrecv(const void* sendbuf, int sendcount, MPI_Datatype sendtype, int dest, int sendtag,
                 void* recvbuf, int recvcount, MPI_Datatype recvtype, int source, int recvtag,
                 MPI_Comm comm, MPI_Status* status) {
  const int rc = MPI_Send(sendbuf, sendcount, sendtype, dest, sendtag, comm);
  return rc != MPI_SUCCESS ? rc : MPI_Recv(recvbuf, recvcount, recvtype, source, recvtag, comm,
                                           status);
}

}  // extern "C"
