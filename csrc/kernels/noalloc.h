/* C interface of the allocation-free paged decode attention entry point (noalloc.cu).
 *
 * This entry point has no counterpart in the reference implementation. It serves callers of this
 * library that must not allocate device memory themselves: hosts whose own memory manager owns
 * the whole device budget and forbids allocations by libraries, and serving loops that must never
 * enter an allocator on their latency-critical path. The kernel's scratch (split-KV partial
 * results) lives in one fixed device array inside the library, so the caller passes only its
 * inputs and its output buffer.
 *
 * Call it from ordinary host code. It makes CUDA runtime calls (device query, symbol lookup,
 * kernel launch), which CUDA forbids inside a host callback or a stream-ordered host function.
 */
#ifndef GOLLEK_NOALLOC_H_
#define GOLLEK_NOALLOC_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
enum {
  GOLLEK_NOALLOC_OK = 0,
  GOLLEK_NOALLOC_ERR_ARGS = 1,        /* null pointer, non-positive size, H not a multiple of Hk */
  GOLLEK_NOALLOC_ERR_SCRATCH = 2,     /* B * H * num_splits * (head_dim + 2) * 4 bytes > capacity */
  GOLLEK_NOALLOC_ERR_CUDA = 3,        /* a CUDA runtime call failed (symbol lookup or launch) */
  GOLLEK_NOALLOC_ERR_UNSUPPORTED = 4  /* block_size != 16, or a head_dim / group pair not built */
};

/* Split-KV paged decode attention without any allocation.
 *   out          [B, H, head_dim] bf16 (written)
 *   q            [B, H, head_dim] bf16, rows q_stride elements apart
 *   cache        [num_blocks, 2, Hk, block_size, head_dim] bf16 (one layer's paged KV)
 *   block_tables [B, bt_stride] int32; seq_lens [B] int32 (KV length of each sequence)
 * head_dim 32, 64, 128 or 256 with H / Hk in {1, 2, 4, 8} (also 16 for head_dim 128);
 * block_size 16. `stream` may be 0. Capacity and sharing of the scratch: see noalloc.cu. */
int gollek_paged_decode_attention_noalloc(void* out, const void* q, int64_t q_stride, const void* cache,
                                          int num_blocks, const int* block_tables, int bt_stride,
                                          const int* seq_lens, int B, int H, int Hk, int head_dim, int block_size,
                                          int num_splits, float scale, cudaStream_t stream);

/* Capacity of the scratch array in bytes. */
size_t gollek_paged_decode_attention_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* GOLLEK_NOALLOC_H_ */
