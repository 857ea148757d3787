/* Randomised traffic through the MPI subset in csrc/mpi_shim, run as several
 * ranks under `torchrun --no-python`. Every rank derives the same message plan
 * from a seed: rounds of messages with random source, destination (self
 * included), tag (from a small set, so tags repeat and interleave) and size
 * (inline slots up to staging segments). Each rank posts its receives and
 * sends of a round as Isend/Irecv in a shuffled order that keeps plan order
 * within every (peer, tag) stream (MPI matches the n-th receive of a stream
 * with the n-th send), completes them with Waitall or a Testall loop, and
 * checks every payload byte. Where a CUDA device is visible, about half of the
 * buffers (chosen per message and side) are device buffers, so host-to-device,
 * device-to-host and device-to-device messages mix with host ones. Prints
 * "rank <r> stress OK <messages> device <0|1>" or "rank <r> FAIL <what>".
 * Arguments: [rounds] [messages per round] [seed]. */
#include <cuda_runtime.h>
#include <mpi.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int rank_, size_;

#define CHECK(cond, what)                                  \
  do {                                                     \
    if (!(cond)) {                                         \
      printf("rank %d FAIL %s\n", rank_, what);            \
      fflush(stdout);                                      \
      MPI_Abort(MPI_COMM_WORLD, 3);                        \
    }                                                      \
  } while (0)

static uint64_t rng_state;
static uint32_t rnd(void) { /* xorshift64* */
  rng_state ^= rng_state >> 12;
  rng_state ^= rng_state << 25;
  rng_state ^= rng_state >> 27;
  return (uint32_t)((rng_state * 2685821657736338717ull) >> 32);
}

typedef struct {
  int src, dst, tag;
  size_t bytes;
  uint32_t salt;
} Msg;

static uint8_t byte_of(const Msg* m, size_t i) {
  return (uint8_t)((i * 131u + m->salt + (uint32_t)m->src * 7u) & 0xffu);
}

int main(int argc, char** argv) {
  const int rounds = argc > 1 ? atoi(argv[1]) : 20;
  const int per_round = argc > 2 ? atoi(argv[2]) : 24;
  const uint64_t seed = argc > 3 ? strtoull(argv[3], NULL, 10) : 1;
  int provided = 0;
  CHECK(MPI_Init_thread(&argc, &argv, MPI_THREAD_FUNNELED, &provided) == MPI_SUCCESS, "init");
  MPI_Comm_rank(MPI_COMM_WORLD, &rank_);
  MPI_Comm_size(MPI_COMM_WORLD, &size_);
  static const size_t sizes[] = {0, 1, 7, 64, 999, 1000, 1001, 4096, 65536, 200003};
  const int nsizes = (int)(sizeof(sizes) / sizeof(sizes[0]));
  Msg* plan = (Msg*)malloc(sizeof(Msg) * (size_t)per_round);
  MPI_Request* reqs = (MPI_Request*)malloc(sizeof(MPI_Request) * 2 * (size_t)per_round);
  uint8_t** bufs = (uint8_t**)calloc(2 * (size_t)per_round, sizeof(uint8_t*));
  int* order = (int*)malloc(sizeof(int) * 2 * (size_t)per_round);
  long checked = 0;
  int ndev = 0;
  const int gpu = cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0;
  if (!gpu) cudaGetLastError();
  else CHECK(cudaSetDevice(rank_ % ndev) == cudaSuccess, "set device");
  uint8_t** devs = (uint8_t**)calloc(2 * (size_t)per_round, sizeof(uint8_t*));
  rng_state = seed * 0x9E3779B97F4A7C15ull + 1;
  for (int round = 0; round < rounds; ++round) {
    for (int i = 0; i < per_round; ++i) {  /* the same plan on every rank */
      plan[i].src = (int)(rnd() % (uint32_t)size_);
      plan[i].dst = (int)(rnd() % (uint32_t)size_);
      plan[i].tag = (int)(rnd() % 3u);
      plan[i].bytes = sizes[rnd() % (uint32_t)nsizes];
      plan[i].salt = rnd();
    }
    const uint32_t mode = rnd() % 2u;  /* 0: Waitall, 1: Testall loop */
    /* this rank's operations: 2i = send of message i, 2i+1 = its receive */
    int nops = 0;
    for (int i = 0; i < per_round; ++i) {
      if (plan[i].src == rank_) order[nops++] = 2 * i;
      if (plan[i].dst == rank_) order[nops++] = 2 * i + 1;
    }
    uint64_t local = rng_state ^ (uint64_t)(rank_ + 1) * 0x632BE59BD9B4E019ull;
    for (int k = nops - 1; k > 0; --k) {  /* rank-local shuffle, plan stream untouched */
      local ^= local << 13;
      local ^= local >> 7;
      local ^= local << 17;
      const int j = (int)(local % (uint64_t)(k + 1));
      const int t = order[k];
      order[k] = order[j];
      order[j] = t;
    }
    /* restore plan order inside each stream: the positions a stream holds in
     * the shuffled order get that stream's operations in plan order */
    for (int k = 0; k < nops; ++k) {
      for (int j = k + 1; j < nops; ++j) {
        const Msg* a = &plan[order[k] / 2];
        const Msg* c = &plan[order[j] / 2];
        const int same = (order[k] % 2 == order[j] % 2) &&
                         (order[k] % 2 == 0 ? a->dst == c->dst : a->src == c->src) &&
                         a->tag == c->tag;
        if (same && order[j] < order[k]) {
          const int t = order[k];
          order[k] = order[j];
          order[j] = t;
        }
      }
    }
    for (int k = 0; k < nops; ++k) {
      const int op = order[k];
      const Msg* m = &plan[op / 2];
      uint8_t* b = (uint8_t*)malloc(m->bytes ? m->bytes : 1);
      bufs[k] = b;
      devs[k] = NULL;
      /* device or host buffer, decided per message and side from its salt */
      const int on_dev = gpu && ((m->salt >> (op % 2 ? 3 : 7)) & 1);
      if (on_dev) CHECK(cudaMalloc((void**)&devs[k], m->bytes ? m->bytes : 1) == cudaSuccess,
                        "cudaMalloc");
      if (op % 2 == 0) {
        for (size_t i = 0; i < m->bytes; ++i) b[i] = byte_of(m, i);
        if (on_dev) CHECK(cudaMemcpy(devs[k], b, m->bytes, cudaMemcpyHostToDevice) == cudaSuccess,
                          "H2D");
        MPI_Isend(on_dev ? devs[k] : b, (int)m->bytes, MPI_BYTE, m->dst, m->tag, MPI_COMM_WORLD,
                  &reqs[k]);
      } else {
        memset(b, 0xEE, m->bytes ? m->bytes : 1);
        if (on_dev) CHECK(cudaMemset(devs[k], 0xEE, m->bytes ? m->bytes : 1) == cudaSuccess,
                          "memset");
        MPI_Irecv(on_dev ? devs[k] : b, (int)m->bytes, MPI_BYTE, m->src, m->tag, MPI_COMM_WORLD,
                  &reqs[k]);
      }
    }
    if (mode == 0) {
      CHECK(MPI_Waitall(nops, reqs, MPI_STATUSES_IGNORE) == MPI_SUCCESS, "waitall");
    } else {
      int flag = 0;
      const double t0 = MPI_Wtime();
      while (!flag) {
        CHECK(MPI_Testall(nops, reqs, &flag, MPI_STATUSES_IGNORE) == MPI_SUCCESS, "testall");
        CHECK(MPI_Wtime() - t0 < 120.0, "testall progress");
      }
    }
    for (int k = 0; k < nops; ++k) {
      const int op = order[k];
      const Msg* m = &plan[op / 2];
      if (op % 2 == 1) {
        if (devs[k])
          CHECK(cudaMemcpy(bufs[k], devs[k], m->bytes, cudaMemcpyDeviceToHost) == cudaSuccess,
                "D2H");
        for (size_t i = 0; i < m->bytes; ++i)
          if (bufs[k][i] != byte_of(m, i)) CHECK(0, "payload");
        ++checked;
      }
      if (devs[k]) cudaFree(devs[k]);
      free(bufs[k]);
    }
  }
  CHECK(MPI_Barrier(MPI_COMM_WORLD) == MPI_SUCCESS, "barrier");
  printf("rank %d stress OK %ld device %d\n", rank_, checked, gpu);
  fflush(stdout);
  free(plan);
  free(reqs);
  free(bufs);
  free(order);
  free(devs);
  MPI_Finalize();
  return 0;
}
