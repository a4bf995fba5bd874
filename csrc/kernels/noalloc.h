/* foa_paged_decode_noalloc: paged decode attention that allocates no device memory.
 *
 * This interface has no counterpart in the reference (furiosa-ai/furiosa-opt-models); it is an
 * addition of this framework, for C callers that cannot allocate device memory while they run: a
 * host runtime with a fixed device-memory budget, code inside another framework's memory pool
 * that forbids foreign allocations, or a plug-in behind a plain C interface with no way to hand
 * back a scratch buffer. They own the inputs and outputs; the working memory for long histories
 * is a fixed array inside the library (FOA_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the
 * library until the process exits).
 *
 * The definition is in noalloc.cu, which includes this header. Plain C compatible.
 */
#ifndef FOA_NOALLOC_H_
#define FOA_NOALLOC_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define FOA_NOALLOC_OK 0
#define FOA_NOALLOC_BAD_ARGUMENT (-2)  /* a null pointer, a non-positive size, head_dim not 64/128 */
#define FOA_NOALLOC_TOO_LARGE (-3)     /* the call needs more than FOA_NOALLOC_SCRATCH_BYTES */
#define FOA_NOALLOC_SETUP_FAILED (-4)  /* no current device, or the array's address lookup failed */
#define FOA_NOALLOC_LAUNCH_FAILED (-5) /* the kernel launch was rejected */

/* Bytes of the library's scratch array: a call needs
 * num_segments * q_heads * ceil(max_keys / keys_per_split) * (head_dim + 1) * 4 bytes, with the
 * log-sum-exp part rounded up to 256 bytes, whenever the histories take more than one split. */
#define FOA_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Decode attention of `num_segments` one-row segments over one layer's paged KV cache.
 *
 * q, o:      BF16 [rows][q_heads][head_dim] on the current device.
 * cache:     the layer's pages; block b holds K[kv_heads][16][head_dim] then V, BF16.
 * table:     int32 block IDs.
 * segments:  int32 [num_segments][5] = row_start, len (must be 1), cached, table_start, nblocks.
 * scale:     softmax scale (1 / sqrt(head_dim) for the usual attention).
 * max_keys:  must bound every segment's history (cached + 1); a longer segment gets zeros in its
 *            output row (it has more splits than the scratch was laid out for).
 * keys_per_split: keys of one split (a multiple of 64); histories longer than one split use the
 *            scratch array.
 * stream:    a cudaStream_t (null: the legacy default stream).
 * error:     optional buffer of `error_len` bytes for a message when the call fails.
 *
 * The first call on each device, with that device current, looks the scratch array's device
 * address up (cudaGetSymbolAddress) and keeps it for the life of the process; make that first
 * call before capturing any stream. A device reset (cudaDeviceReset) or a destroyed and re-created
 * primary context invalidates the kept address: do not call this entry point afterwards.
 *
 * Every call on a device shares the one array, which keeps the last call's contents (each call
 * writes every partial before reading it). Calls whose kernels overlap on the GPU, from unordered
 * streams or several host threads, race on the array: order them on one stream.
 *
 * Returns FOA_NOALLOC_OK, or a negative code (nothing launched) with a message in `error`. */
int foa_paged_decode_noalloc(const void* q, void* o, const void* cache, const int32_t* table,
                             const int32_t* segments, int num_segments, int q_heads, int kv_heads,
                             int head_dim, float scale, int max_keys, int keys_per_split, void* stream,
                             char* error, int error_len);

#ifdef __cplusplus
}
#endif

#endif /* FOA_NOALLOC_H_ */
