/* Allocation-free entry point of the paged decode attention kernel.
 *
 * This entry point has no counterpart in the reference (everserve-ai/everserve); it is an
 * addition of this library.
 *
 * Who it is for: callers that cannot allocate device memory when they call the kernel. Typical
 * cases are host programs that reserve all device memory at start-up and hand it out from their
 * own pools (so a cudaMalloc later would fail or break their accounting), runtimes that run under
 * a hard memory cap, and latency-critical paths where an allocation may block on the driver. The
 * regular binding (everserve_b200._C.paged_decode) needs its split-KV scratch passed in, which the
 * Python side allocates through torch; this entry point instead uses a fixed scratch area that is
 * part of the library itself.
 *
 * Scratch: a file-scope `static __device__` array of ES_NOALLOC_SCRATCH_BYTES bytes (8.25 MiB plus
 * a status word and 16 KiB of split tickets, which start at zero and which every call leaves at
 * zero) in attention.cu. Every GPU that loads the library holds that array until the
 * process exits. Requests whose split-KV partials do not fit are rejected (return value
 * cudaErrorInvalidValue, and es_noalloc_last_error() says why); nothing is allocated to make them
 * fit. The caller still passes every input and output buffer.
 *
 * Set-up: the first call on a device looks up the array's device address with
 * cudaGetSymbolAddress, with that device current, and remembers it for the device. Make that first
 * call (or call es_noalloc_setup) on each device before any stream capture starts.
 *
 * Sharing: every call on a device uses the same scratch array, which keeps the last call's
 * contents. Each call clears the status word it needs at zero; calls whose kernels overlap on the
 * GPU (two streams, or two host threads) race on the scratch and must be serialised by the caller.
 *
 * Layouts are those of the regular binding: q [batch, q_heads, head_dim] bf16 (rows of q_stride
 * elements), cache [num_blocks, 2, kv_heads, block_size, head_dim] bf16 contiguous, block_tables
 * [batch, *] int32 (rows of bt_stride), ctx_lens [batch] int32, out [batch, q_heads * head_dim]
 * bf16 (rows of out_stride). Positions are split into runs of 256, so the result matches the
 * regular entry point's bit for bit when that one is given the same split length.
 *
 * Limits of the inputs: batch * kv_heads at most ES_NOALLOC_TICKETS; every ctx_lens[b] must be at
 * most max_model_len (the scratch and the grid
 * are sized from max_model_len, so positions past it would be left out of the result), and each
 * row of block_tables must hold at least ceil(ctx_lens[b] / block_size) valid block indices.
 */
#ifndef ES_NOALLOC_H_
#define ES_NOALLOC_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ES_NOALLOC_PART_FLOATS (1 << 21) /* split partial outputs: batch * q_heads * splits * head_dim */
#define ES_NOALLOC_ML_FLOATS (1 << 16)   /* split maxima and sums: batch * q_heads * splits * 2 */
#define ES_NOALLOC_TICKETS 4096          /* split tickets, one per (sequence, kv head): batch * kv_heads */

/* Look up the scratch array's address on the current device (idempotent). Returns a cudaError_t. */
int es_noalloc_setup(void);

/* Paged decode attention with the library's own scratch; `stream` is a cudaStream_t (NULL for the
 * default stream). Returns 0 (cudaSuccess) or a cudaError_t value. */
int es_paged_decode_noalloc(const void* q, int64_t q_stride, const void* cache, int64_t num_blocks, int kv_heads,
                            int block_size, int head_dim, const int* block_tables, int64_t bt_stride,
                            const int* ctx_lens, void* out, int64_t out_stride, int batch, int q_heads,
                            int max_model_len, float scale, void* stream);

/* Copy the last call's status word to *status (0: every bounded wait completed). Synchronises the
 * stream. Returns a cudaError_t. */
int es_noalloc_status(void* stream, int* status);

/* Why the last rejected call was rejected (a static string; empty when none was). */
const char* es_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* ES_NOALLOC_H_ */
