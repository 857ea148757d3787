/* A subset of the MPI C interface (MPI standard 3.1 names and signatures), for
 * building the reference prototype's benchmarks unmodified on machines without
 * an MPI installation. Ranks and the rendezvous come from torchrun-style
 * environment variables (RANK, WORLD_SIZE, MASTER_ADDR, MASTER_PORT); messages
 * travel through a TCP key-value store, and buffers in device memory are staged
 * through host memory (CUDA-aware semantics). One communicator (the world) and
 * the point-to-point, barrier, broadcast and reduce calls the benchmarks use,
 * plus allreduce, gather, allgather and scatter. */
#ifndef MGFA_MPI_SHIM_H
#define MGFA_MPI_SHIM_H

#ifdef __cplusplus
extern "C" {
#endif

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
typedef int MPI_Info;
typedef struct mgfa_mpi_request* MPI_Request;

typedef struct {
  int MPI_SOURCE;
  int MPI_TAG;
  int MPI_ERROR;
  int count_bytes;
} MPI_Status;

#define MPI_SUCCESS 0
#define MPI_ERR_OTHER 15

#define MPI_COMM_WORLD ((MPI_Comm)1)
#define MPI_COMM_NULL ((MPI_Comm)0)
#define MPI_INFO_NULL ((MPI_Info)0)
#define MPI_COMM_TYPE_SHARED 1

#define MPI_BYTE ((MPI_Datatype)1)
#define MPI_CHAR ((MPI_Datatype)2)
#define MPI_INT ((MPI_Datatype)3)
#define MPI_FLOAT ((MPI_Datatype)4)
#define MPI_DOUBLE ((MPI_Datatype)5)

#define MPI_MAX ((MPI_Op)1)
#define MPI_MIN ((MPI_Op)2)
#define MPI_SUM ((MPI_Op)3)

#define MPI_THREAD_SINGLE 0
#define MPI_THREAD_FUNNELED 1
#define MPI_THREAD_SERIALIZED 2
#define MPI_THREAD_MULTIPLE 3

#define MPI_STATUS_IGNORE ((MPI_Status*)0)
#define MPI_STATUSES_IGNORE ((MPI_Status*)0)
#define MPI_REQUEST_NULL ((MPI_Request)0)

int MPI_Init(int* argc, char*** argv);
int MPI_Init_thread(int* argc, char*** argv, int required, int* provided);
int MPI_Finalize(void);
int MPI_Abort(MPI_Comm comm, int errorcode);
int MPI_Comm_rank(MPI_Comm comm, int* rank);
int MPI_Comm_size(MPI_Comm comm, int* size);
int MPI_Comm_split_type(MPI_Comm comm, int split_type, int key, MPI_Info info,
                        MPI_Comm* newcomm);
int MPI_Comm_free(MPI_Comm* comm);
double MPI_Wtime(void);

int MPI_Type_size(MPI_Datatype datatype, int* size);
int MPI_Get_count(const MPI_Status* status, MPI_Datatype datatype, int* count);

int MPI_Barrier(MPI_Comm comm);
int MPI_Bcast(void* buffer, int count, MPI_Datatype datatype, int root, MPI_Comm comm);
int MPI_Reduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype, MPI_Op op,
               int root, MPI_Comm comm);
int MPI_Allreduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype,
                  MPI_Op op, MPI_Comm comm);
int MPI_Gather(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
               int recvcount, MPI_Datatype recvtype, int root, MPI_Comm comm);
int MPI_Allgather(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
                  int recvcount, MPI_Datatype recvtype, MPI_Comm comm);
int MPI_Scatter(const void* sendbuf, int sendcount, MPI_Datatype sendtype, void* recvbuf,
                int recvcount, MPI_Datatype recvtype, int root, MPI_Comm comm);

int MPI_Send(const void* buf, int count, MPI_Datatype datatype, int dest, int tag,
             MPI_Comm comm);
int MPI_Recv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
             MPI_Status* status);
int MPI_Sendrecv(const void* sendbuf, int sendcount, MPI_Datatype sendtype, int dest, int sendtag,
                 void* recvbuf, int recvcount, MPI_Datatype recvtype, int source, int recvtag,
                 MPI_Comm comm, MPI_Status* status);
int MPI_Isend(const void* buf, int count, MPI_Datatype datatype, int dest, int tag,
              MPI_Comm comm, MPI_Request* request);
int MPI_Irecv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
              MPI_Request* request);
int MPI_Wait(MPI_Request* request, MPI_Status* status);
int MPI_Waitall(int count, MPI_Request array_of_requests[], MPI_Status array_of_statuses[]);
int MPI_Testall(int count, MPI_Request array_of_requests[], int* flag,
                MPI_Status array_of_statuses[]);

#ifdef __cplusplus
}
#endif

#endif /* MGFA_MPI_SHIM_H */
