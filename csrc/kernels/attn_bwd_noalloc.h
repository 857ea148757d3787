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

/* Size of the static scratch array (36 MiB). A call needs
 *   256 + 2 * 4 * ceil(max(seqlen_q, seqlen_k) / 128) * 4
 *   + 2 * 4 * batch * heads_q * ceil(seqlen_q / 128) * 128   bytes
 * (e.g. batch 1, 32 query heads, 128K tokens fits). */
#define MGFA_BWD_NOALLOC_SCRATCH_BYTES (36u * 1024u * 1024u)

/* Return codes. */
#define MGFA_NOALLOC_OK 0
#define MGFA_NOALLOC_BAD_ARGUMENT 1   /* null pointer, bad shape or alignment */
#define MGFA_NOALLOC_TOO_LARGE 2      /* problem needs more scratch than the static array */
#define MGFA_NOALLOC_CUDA_ERROR 3     /* set-up or launch failed; details on stderr */

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
 * called. The first call on a device looks up that device's scratch address
 * (cudaGetSymbolAddress with the device current) and caches it; make that first
 * call before any stream capture on the device.
 *
 * Every call on a device shares the same scratch array, which keeps the last
 * call's contents. Calls whose work overlaps on the GPU (different streams
 * without ordering, or different host threads) race on the scratch and give
 * wrong results: order them on one stream or synchronise between them.
 */
int mgfa_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                          const void* out, const float* lse, float* dq, float* dk, float* dv,
                          int batch, int seqlen_q, int seqlen_k, int heads_q, int heads_kv,
                          float softmax_scale, int causal, void* stream);

#ifdef __cplusplus
}
#endif

#endif
