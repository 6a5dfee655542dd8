/* Allocation-free entry points of the bloom_b200 CUDA library (bloom_b200/_C*.so).
 *
 * This API has no counterpart in the reference; it is an addition of this
 * library for callers that cannot allocate GPU memory when they call in: a
 * host application that fixed its memory budget at start-up and forbids
 * cudaMalloc afterwards, code running on a stream whose memory pool belongs
 * to another framework, or a C program that loads the library without
 * PyTorch and so has no caching allocator to take scratch from.
 *
 * The scratch these functions need lives in a fixed 8 MiB array inside the
 * library (one per GPU, held until the process exits).  See
 * csrc/kernels/attention.cu for the full contract: the first call on a device
 * does per-device set-up and should come before any stream capture; calls
 * that overlap on the GPU share the scratch and race; requests that do not
 * fit return BLOOM_NOALLOC_TOO_LARGE.
 */
#ifndef BLOOM_NOALLOC_H
#define BLOOM_NOALLOC_H

#ifdef __cplusplus
extern "C" {
#endif

#define BLOOM_NOALLOC_OK 0
#define BLOOM_NOALLOC_BAD_ARGUMENT -1
#define BLOOM_NOALLOC_TOO_LARGE -2
#define BLOOM_NOALLOC_CUDA_ERROR -3
#define BLOOM_NOALLOC_TENSOR_MAP_ERROR -4
#define BLOOM_NOALLOC_LAUNCH_ERROR -5

/* Paged decode / verify attention (GQA, causal over the last q_len tokens).
 *   q          [batch * q_len, num_q_heads, 128] bf16 (device)
 *   out        [batch * q_len, num_q_heads, 128] bf16 (device)
 *   kv_layer   one layer of the paged cache, [num_blocks, 2, num_kv_heads, 16, 128] bf16 (device)
 *   block_table [batch, block_table_stride] int32 page ids (device)
 *   seq_lens   [batch] int32 kv lengths including the q_len new tokens (device)
 *   splits     split-K factor over the context; > 1 uses the library's scratch
 *   stream     cudaStream_t (NULL = legacy default stream)
 * Returns BLOOM_NOALLOC_OK or a negative code; the kernel is only queued. */
int bloom_paged_decode_attention_noalloc(const void* q, void* out, const void* kv_layer, long long num_blocks,
                                         int num_q_heads, int num_kv_heads, const int* block_table,
                                         int block_table_stride, const int* seq_lens, int batch, int q_len,
                                         int splits, float scale, void* stream);

/* Reads and clears the status word of the current device.  Synchronous: it
 * waits for all work on the device first (every stream), so the bits of a
 * call queued on a non-blocking stream are included.  Not during capture. */
int bloom_noalloc_status(int* bits);

#ifdef __cplusplus
}
#endif

#endif /* BLOOM_NOALLOC_H */
