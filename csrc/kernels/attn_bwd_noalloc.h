/* Allocation-free attention backward: C entry point.
 *
 * This interface has no counterpart in the reference prototype; it exists for
 * callers that must not allocate device memory, for example code running
 * inside a custom memory-pool or graph-building framework that forbids
 * cudaMalloc/cudaFree, or a host runtime that owns every device allocation
 * itself and only hands out input/output buffers.
 *
 * The backward needs two per-row scratch vectors (the LSE in log2 units and
 * delta = rowsum(dO * O)), a kernel status word and the causal tile positions.
 * Here they live in one statically sized device array inside this library
 * (MGFA_BWD_NOALLOC_SCRATCH_BYTES per GPU, kept for the life of the process on
 * every GPU that loads the library) instead of in memory the call allocates.
 */
#ifndef MGFA_ATTN_BWD_NOALLOC_H
#define MGFA_ATTN_BWD_NOALLOC_H

#ifdef __cplusplus
extern "C" {
#endif

/* Size of the static scratch array (36 MiB). With round256(x) = x rounded up
 * to a multiple of 256, n_q_tiles = ceil(seqlen_q / 128) and
 * n_kv_tiles = ceil(seqlen_k / 128), a call needs exactly
 *   256                                              (status word, padded)
 *   + round256(4 * (n_q_tiles + n_kv_tiles))         (causal tile positions)
 *   + 2 * round256(4 * batch * heads_q * n_q_tiles * 128)   (lse2 and delta)
 * bytes, and is rejected with MGFA_NOALLOC_TOO_LARGE above the array's size.
 * So batch * heads_q * n_q_tiles * 128 may reach about 4.7 million rows
 * (e.g. batch 1, 32 query heads, 128K tokens fits). */
#define MGFA_BWD_NOALLOC_SCRATCH_BYTES (36u * 1024u * 1024u)

/* Return codes. */
#define MGFA_NOALLOC_OK 0
#define MGFA_NOALLOC_BAD_ARGUMENT 1   /* null pointer, bad shape or alignment */
#define MGFA_NOALLOC_TOO_LARGE 2      /* problem needs more scratch than the static array */
#define MGFA_NOALLOC_CUDA_ERROR 3     /* set-up or launch failed, or a CUDA error was
                                         already pending on entry (left in place for its
                                         owner); details on stderr */

/* Gradients of softmax(scale * Q K^T) V for contiguous tensors on the current
 * device:
 *   dout, q, out : bf16 [batch, seqlen_q, heads_q, 128]
 *   k, v         : bf16 [batch, seqlen_k, heads_kv, 128]
 *   lse          : fp32 [batch, heads_q, seqlen_q], natural-log LSE of the forward
 *   dq           : fp32 [batch, seqlen_q, heads_q, 128]   (written)
 *   dk, dv       : fp32 [batch, seqlen_k, heads_kv, 128]  (written)
 *   causal       : 0 or 1 (query i sees keys 0..i)
 *   stream       : cudaStream_t (NULL = legacy default stream)
 * All work is enqueued on `stream`; the call returns before it finishes.
 *
 * No device memory is allocated or freed, and no allocating library routine is
 * called. The scratch address of a device is looked up with
 * cudaGetSymbolAddress (with that device current) on every call made outside
 * stream capture, so a call after a device reset finds the reloaded array; a
 * call under capture reuses the address of the last call made outside capture
 * on that device. So make the first call on each device before any stream
 * capture on it (a first call under capture is rejected with
 * MGFA_NOALLOC_CUDA_ERROR).
 *
 * Every call on a device shares the same scratch array, which keeps the last
 * call's contents. Calls whose work overlaps on the GPU (different streams
 * without ordering, or different host threads) race on the scratch and give
 * wrong results: order them on one stream or synchronise between them.
 *
 * A return of MGFA_NOALLOC_OK means the work was enqueued. Whether the kernels
 * finished their work is in the status word that they leave in the scratch
 * array: read it with mgfa_attn_bwd_noalloc_status() below.
 */
int mgfa_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                          const void* out, const float* lse, float* dq, float* dk, float* dv,
                          int batch, int seqlen_q, int seqlen_k, int heads_q, int heads_kv,
                          float softmax_scale, int causal, void* stream);

/* Copies the status word of the last mgfa_attn_bwd_noalloc() call on the
 * current device into *host_status, enqueued on `stream` (use the stream of
 * that call). It allocates nothing. Synchronise the stream before reading
 * *host_status (with pageable host memory the copy itself waits for the
 * stream). 0 means the kernels ran to completion; any other value means a
 * bounded wait inside a kernel gave up (code in bits 0-7, site in bits 8-15)
 * and dq, dk and dv may be partly written. Returns MGFA_NOALLOC_OK, or
 * MGFA_NOALLOC_CUDA_ERROR when the copy could not be enqueued (or no call was
 * made on this device yet). */
int mgfa_attn_bwd_noalloc_status(unsigned int* host_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif
