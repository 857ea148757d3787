/* Semantics check of the MPI subset in csrc/mpi_shim, run as several ranks
 * under `torchrun --no-python`. Prints "rank <r> OK" or "rank <r> FAIL <what>"
 * and exits non-zero on the first failed check. Covers: message order per
 * (source, tag), tags that overtake each other, Isend/Irecv with Waitall and
 * Testall, Sendrecv around the ring, Bcast from a non-zero root, Reduce
 * (MAX, MIN, SUM over double, float and int), Allreduce, Gather, Allgather,
 * Scatter, Get_count and Type_size, Barrier, the shared-memory
 * split and Wtime; more sends in flight than a mailbox holds, a payload
 * larger than a mailbox slot, and repeated barriers. Rank 0 also prints the
 * host round-trip latency between ranks 0 and 1 ("latency_us <x>") and the
 * one-way rate of 16 MB host messages between them ("bulk_GBps <x>").
 * Where a CUDA device is visible, the device section sends cudaMalloc'd
 * buffers (CUDA IPC in the shim) around the ring, from an interior pointer
 * and with Sendrecv and Isend/Irecv, and prints "rank <r> device OK";
 * otherwise "rank <r> device skipped". Ranks share the visible devices
 * round-robin. */
#include <cuda_runtime.h>
#include <mpi.h>
#include <stdio.h>
#include <stdlib.h>

static int rank_, size_;

#define CHECK(cond, what)                                         \
  do {                                                            \
    if (!(cond)) {                                                \
      printf("rank %d FAIL %s\n", rank_, what);                   \
      fflush(stdout);                                             \
      MPI_Abort(MPI_COMM_WORLD, 3);                               \
    }                                                             \
  } while (0)

int main(int argc, char** argv) {
  int provided = -1;
  CHECK(MPI_Init_thread(&argc, &argv, MPI_THREAD_FUNNELED, &provided) == MPI_SUCCESS, "init");
  CHECK(provided >= MPI_THREAD_FUNNELED, "thread level");
  MPI_Comm_rank(MPI_COMM_WORLD, &rank_);
  MPI_Comm_size(MPI_COMM_WORLD, &size_);
  const int right = (rank_ + 1) % size_, left = (rank_ - 1 + size_) % size_;

  /* shared-memory split: one node, so the local rank is the world rank */
  MPI_Comm local;
  int lr = -1, ls = -1;
  MPI_Comm_split_type(MPI_COMM_WORLD, MPI_COMM_TYPE_SHARED, 0, MPI_INFO_NULL, &local);
  MPI_Comm_rank(local, &lr);
  MPI_Comm_size(local, &ls);
  MPI_Comm_free(&local);
  CHECK(lr == rank_ && ls == size_, "split_type");

  /* three messages with tag 7 then one with tag 9: a receive of tag 9 posted
   * first must get the tag-9 message, and tag-7 messages arrive in order */
  double a[3][4], b[4];
  for (int m = 0; m < 3; ++m)
    for (int i = 0; i < 4; ++i) a[m][i] = rank_ * 100 + m * 10 + i;
  for (int i = 0; i < 4; ++i) b[i] = -(rank_ * 100 + i);
  for (int m = 0; m < 3; ++m) MPI_Send(a[m], 4, MPI_DOUBLE, right, 7, MPI_COMM_WORLD);
  MPI_Send(b, 4, MPI_DOUBLE, right, 9, MPI_COMM_WORLD);
  double rb[4];
  MPI_Status st;
  MPI_Recv(rb, 4, MPI_DOUBLE, left, 9, MPI_COMM_WORLD, &st);
  CHECK(st.MPI_SOURCE == left && st.MPI_TAG == 9, "status");
  for (int i = 0; i < 4; ++i) CHECK(rb[i] == -(left * 100 + i), "tag 9 payload");
  for (int m = 0; m < 3; ++m) {
    MPI_Recv(rb, 4, MPI_DOUBLE, left, 7, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
    for (int i = 0; i < 4; ++i) CHECK(rb[i] == left * 100 + m * 10 + i, "tag 7 order");
  }

  /* nonblocking pair, completed by Testall (polled) then Waitall */
  float sendf[8], recvf[8];
  for (int i = 0; i < 8; ++i) sendf[i] = (float)(rank_ * 8 + i);
  MPI_Request req[2];
  MPI_Irecv(recvf, 8, MPI_FLOAT, left, 3, MPI_COMM_WORLD, &req[0]);
  MPI_Isend(sendf, 8, MPI_FLOAT, right, 3, MPI_COMM_WORLD, &req[1]);
  int flag = 0;
  const double t0 = MPI_Wtime();
  while (!flag && MPI_Wtime() - t0 < 60.0)
    MPI_Testall(2, req, &flag, MPI_STATUSES_IGNORE);
  CHECK(flag, "testall");
  CHECK(req[0] == MPI_REQUEST_NULL && req[1] == MPI_REQUEST_NULL, "requests freed");
  for (int i = 0; i < 8; ++i) CHECK(recvf[i] == (float)(left * 8 + i), "isend payload");
  MPI_Irecv(recvf, 8, MPI_FLOAT, left, 4, MPI_COMM_WORLD, &req[0]);
  MPI_Isend(sendf, 8, MPI_FLOAT, right, 4, MPI_COMM_WORLD, &req[1]);
  MPI_Waitall(2, req, MPI_STATUSES_IGNORE);
  for (int i = 0; i < 8; ++i) CHECK(recvf[i] == (float)(left * 8 + i), "waitall payload");

  /* ring rotation with Sendrecv: after size steps every rank holds its own value */
  int token = rank_, got = -1;
  for (int s = 0; s < size_; ++s) {
    MPI_Sendrecv(&token, 1, MPI_INT, right, 0, &got, 1, MPI_INT, left, 0, MPI_COMM_WORLD,
                 MPI_STATUS_IGNORE);
    token = got;
  }
  CHECK(token == rank_, "sendrecv ring");

  /* a message to itself */
  int self_out = 42 + rank_, self_in = -1;
  MPI_Sendrecv(&self_out, 1, MPI_INT, rank_, 30, &self_in, 1, MPI_INT, rank_, 30, MPI_COMM_WORLD,
               MPI_STATUS_IGNORE);
  CHECK(self_in == 42 + rank_, "self message");

  /* broadcast from the last rank */
  char id[16];
  for (int i = 0; i < 16; ++i) id[i] = (char)(rank_ == size_ - 1 ? 'a' + i : 0);
  MPI_Bcast(id, 16, MPI_BYTE, size_ - 1, MPI_COMM_WORLD);
  for (int i = 0; i < 16; ++i) CHECK(id[i] == 'a' + i, "bcast");

  /* reductions to root 0 */
  double dv[2] = {(double)rank_, -(double)rank_}, dmax[2] = {0, 0};
  MPI_Reduce(dv, dmax, 2, MPI_DOUBLE, MPI_MAX, 0, MPI_COMM_WORLD);
  float fv = (float)(rank_ + 1), fmin = 0;
  MPI_Reduce(&fv, &fmin, 1, MPI_FLOAT, MPI_MIN, 0, MPI_COMM_WORLD);
  int iv = rank_ + 1, isum = 0;
  MPI_Reduce(&iv, &isum, 1, MPI_INT, MPI_SUM, 0, MPI_COMM_WORLD);
  if (rank_ == 0) {
    CHECK(dmax[0] == size_ - 1 && dmax[1] == 0.0, "reduce max");
    CHECK(fmin == 1.0f, "reduce min");
    CHECK(isum == size_ * (size_ + 1) / 2, "reduce sum");
  }

  /* allreduce, gather (to the last rank), allgather, scatter (from rank 0), counts */
  double sin3[3] = {(double)rank_, 2.0 * rank_, 1.0}, sout3[3] = {0, 0, 0};
  MPI_Allreduce(sin3, sout3, 3, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
  CHECK(sout3[0] == size_ * (size_ - 1) / 2.0 && sout3[1] == 2.0 * sout3[0] &&
            sout3[2] == (double)size_, "allreduce");
  int mine[2] = {rank_ * 10, rank_ * 10 + 1};
  int* allv = (int*)malloc(2 * (size_t)size_ * sizeof(int));
  MPI_Allgather(mine, 2, MPI_INT, allv, 2, MPI_INT, MPI_COMM_WORLD);
  for (int r = 0; r < size_; ++r)
    CHECK(allv[2 * r] == r * 10 && allv[2 * r + 1] == r * 10 + 1, "allgather");
  for (int i = 0; i < 2 * size_; ++i) allv[i] = -1;
  MPI_Gather(mine, 2, MPI_INT, allv, 2, MPI_INT, size_ - 1, MPI_COMM_WORLD);
  if (rank_ == size_ - 1)
    for (int r = 0; r < size_; ++r) CHECK(allv[2 * r] == r * 10, "gather");
  for (int i = 0; i < 2 * size_; ++i) allv[i] = 100 + i;
  int part[2] = {-1, -1};
  MPI_Scatter(allv, 2, MPI_INT, part, 2, MPI_INT, 0, MPI_COMM_WORLD);
  CHECK(part[0] == 100 + 2 * rank_ && part[1] == 101 + 2 * rank_, "scatter");
  free(allv);
  int cnt = -1, tsz = -1;
  MPI_Get_count(&st, MPI_DOUBLE, &cnt);
  MPI_Type_size(MPI_DOUBLE, &tsz);
  CHECK(cnt == 4 && tsz == 8, "counts");

  /* more sends in flight than a mailbox has slots: the excess wait in the
   * sender's queue until the receiver frees slots */
  enum { kMany = 40 };
  int many_out[kMany], many_in[kMany];
  MPI_Request mreq[2 * kMany];
  for (int m = 0; m < kMany; ++m) {
    many_out[m] = rank_ * 1000 + m;
    MPI_Isend(&many_out[m], 1, MPI_INT, right, 11, MPI_COMM_WORLD, &mreq[m]);
  }
  for (int m = 0; m < kMany; ++m)
    MPI_Irecv(&many_in[m], 1, MPI_INT, left, 11, MPI_COMM_WORLD, &mreq[kMany + m]);
  MPI_Waitall(2 * kMany, mreq, MPI_STATUSES_IGNORE);
  for (int m = 0; m < kMany; ++m) CHECK(many_in[m] == left * 1000 + m, "queued sends");

  /* a payload larger than a slot */
  enum { kBig = 300000 };
  float* bo = (float*)malloc(kBig * sizeof(float));
  float* bi = (float*)malloc(kBig * sizeof(float));
  for (int i = 0; i < kBig; ++i) bo[i] = (float)(rank_ * 7 + i % 1000);
  MPI_Sendrecv(bo, kBig, MPI_FLOAT, right, 12, bi, kBig, MPI_FLOAT, left, 12, MPI_COMM_WORLD,
               MPI_STATUS_IGNORE);
  for (int i = 0; i < kBig; ++i) CHECK(bi[i] == (float)(left * 7 + i % 1000), "large payload");
  free(bo);
  free(bi);

  for (int i = 0; i < 200; ++i) CHECK(MPI_Barrier(MPI_COMM_WORLD) == MPI_SUCCESS, "barrier");

  /* host round trip between ranks 0 and 1 */
  if (rank_ < 2) {
    const int peer = 1 - rank_, n = 2000;
    double v = 0.0;
    const double ts = MPI_Wtime();
    for (int i = 0; i < n; ++i) {
      if (rank_ == 0) {
        MPI_Send(&v, 1, MPI_DOUBLE, peer, 13, MPI_COMM_WORLD);
        MPI_Recv(&v, 1, MPI_DOUBLE, peer, 13, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
      } else {
        MPI_Recv(&v, 1, MPI_DOUBLE, peer, 13, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
        v += 1.0;
        MPI_Send(&v, 1, MPI_DOUBLE, peer, 13, MPI_COMM_WORLD);
      }
    }
    if (rank_ == 0) {
      CHECK(v == (double)n, "ping-pong");
      printf("latency_us %.2f\n", (MPI_Wtime() - ts) / n * 1e6);
    }
    /* 16 MB messages, bounced back and forth: one-way bytes per second */
    const size_t nb = (size_t)16 << 20;
    const int reps = 10;
    char* big = (char*)malloc(nb);
    for (size_t i = 0; i < nb; ++i) big[i] = (char)(i * 7 + 3);
    const double tb = MPI_Wtime();
    for (int i = 0; i < reps; ++i) {
      if (rank_ == 0) {
        MPI_Send(big, (int)nb, MPI_BYTE, peer, 14, MPI_COMM_WORLD);
        MPI_Recv(big, (int)nb, MPI_BYTE, peer, 14, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
      } else {
        MPI_Recv(big, (int)nb, MPI_BYTE, peer, 14, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
        MPI_Send(big, (int)nb, MPI_BYTE, peer, 14, MPI_COMM_WORLD);
      }
    }
    for (size_t i = 0; i < nb; i += 4099) CHECK(big[i] == (char)(i * 7 + 3), "bulk payload");
    if (rank_ == 0) printf("bulk_GBps %.2f\n", 2.0 * reps * nb / (MPI_Wtime() - tb) / 1e9);
    free(big);
  }

  /* device buffers */
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0) {
    CHECK(cudaSetDevice(rank_ % ndev) == cudaSuccess, "set device");
    enum { kN = 1 << 20, kOff = 1234 };
    float *d_a = NULL, *d_b = NULL;
    CHECK(cudaMalloc((void**)&d_a, (kN + kOff) * sizeof(float)) == cudaSuccess, "malloc");
    CHECK(cudaMalloc((void**)&d_b, kN * sizeof(float)) == cudaSuccess, "malloc");
    float* h = (float*)malloc(kN * sizeof(float));
    for (int i = 0; i < kN; ++i) h[i] = (float)(rank_ * 4096 + i % 4096);
    CHECK(cudaMemcpy(d_a + kOff, h, kN * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess,
          "H2D");
    /* rotate the buffer once around the ring; step s holds rank (r - s - 1)'s data */
    float* cur = d_a + kOff;  /* an interior pointer of its allocation */
    float* nxt = d_b;
    for (int s = 0; s < size_; ++s) {
      const int owner = (rank_ - s - 1 + 2 * size_) % size_;
      if (s % 2 == 0) {
        MPI_Sendrecv(cur, kN, MPI_FLOAT, right, 20 + s, nxt, kN, MPI_FLOAT, left, 20 + s,
                     MPI_COMM_WORLD, MPI_STATUS_IGNORE);
      } else {
        MPI_Request dr[2];
        MPI_Irecv(nxt, kN, MPI_FLOAT, left, 20 + s, MPI_COMM_WORLD, &dr[0]);
        MPI_Isend(cur, kN, MPI_FLOAT, right, 20 + s, MPI_COMM_WORLD, &dr[1]);
        MPI_Waitall(2, dr, MPI_STATUSES_IGNORE);
      }
      CHECK(cudaMemcpy(h, nxt, kN * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess,
            "D2H");
      for (int i = 0; i < kN; i += 997)
        CHECK(h[i] == (float)(owner * 4096 + i % 4096), "device payload");
      float* t = cur;
      cur = nxt;
      nxt = t;
    }
    /* a device message to itself (the ring left other ranks' data in d_a) */
    for (int i = 0; i < kN; ++i) h[i] = (float)(rank_ * 4096 + i % 4096);
    CHECK(cudaMemcpy(d_a + kOff, h, kN * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess,
          "H2D");
    MPI_Sendrecv(d_a + kOff, kN, MPI_FLOAT, rank_, 40, d_b, kN, MPI_FLOAT, rank_, 40,
                 MPI_COMM_WORLD, MPI_STATUS_IGNORE);
    CHECK(cudaMemcpy(h, d_b, kN * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess, "D2H");
    for (int i = 0; i < kN; i += 997)
      CHECK(h[i] == (float)(rank_ * 4096 + i % 4096), "device self message");
    cudaFree(d_a);
    cudaFree(d_b);
    free(h);
    printf("rank %d device OK\n", rank_);
  } else {
    cudaGetLastError();
    printf("rank %d device skipped\n", rank_);
  }

  MPI_Barrier(MPI_COMM_WORLD);
  CHECK(MPI_Wtime() >= t0, "wtime");
  printf("rank %d OK\n", rank_);
  fflush(stdout);
  MPI_Finalize();
  return 0;
}
