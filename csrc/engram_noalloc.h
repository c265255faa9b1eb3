/* Public C interface of the allocation-free per-owner request pack.
 *
 * This entry point has no counterpart in the reference.  It is for callers
 * that cannot allocate GPU memory themselves: code that runs while a stream is
 * being captured into a CUDA Graph (cudaMalloc is not allowed there), plugins
 * inside a host framework that owns every device allocation through its own
 * pool, and plain C callers that link this library without torch and its
 * caching allocator.  The caller passes the indices and both outputs; the
 * kernel's scratch (slot cursors and arrival counters) is a file-scope device
 * array of ENGRAM_NOALLOC_SCRATCH_BYTES inside the library, which every GPU
 * that loads the library keeps until the process exits.
 *
 * What it computes: the non-padding requests of `indices` ([layers][tokens *
 * ept] int32 on the current device) are bucketed by owner o = x / entries[l]:
 *     packed[o][l][i] = (position << 32) | (table_base[l] + x % entries[l])
 * for i < counts[l][o], where position is the flat token * ept + slot index,
 * table_base[l] is the sum of entries[0..l), and only owners with
 * owners_host[o] != 0 are packed.  `packed` is int64 [world][layers][capacity]
 * and `counts` int32 [layers][world], both device memory.  The order of the
 * entries of one owner is not specified.  Negative ids are padding.  Ids at or
 * beyond world * entries[l] are skipped without an error: they appear in no
 * owner's list and in no count.
 *
 * Limits: layers <= ENGRAM_NOALLOC_MAX_LAYERS, world <= ENGRAM_NOALLOC_MAX_OWNERS,
 * tokens * ept <= capacity, tokens * ept * layers < 2^32, world * entries[l] < 2^31,
 * and the sum of entries below 2^32.  A call beyond them returns a nonzero
 * code with a message and launches nothing.
 *
 * Set-up: the first call on a device, with that device current, looks up the
 * array's device address with cudaGetSymbolAddress and caches it per device.
 * Make that first call before any stream capture begins.  The cached address
 * assumes the device is not reset (cudaDeviceReset) while the library is
 * loaded.
 *
 * Sharing: all calls on a device use the same array, which keeps the last
 * call's contents.  Each call clears the cursors and counters on the caller's
 * stream before its kernel, so calls ordered on one stream (or otherwise
 * serialised) are correct.  Calls that overlap on the GPU, for example on two
 * unsynchronised streams, race on the array and give wrong results.
 *
 * The entry point calls no allocating routine (no cudaMalloc, no cudaFree, no
 * torch allocation): only cudaGetSymbolAddress (once per device),
 * cudaMemsetAsync on the array or on `counts`, and the kernel launch.
 */
#ifndef ENGRAM_NOALLOC_H
#define ENGRAM_NOALLOC_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#define ENGRAM_NOALLOC_SCRATCH_BYTES 32768
#define ENGRAM_NOALLOC_MAX_LAYERS 32
#define ENGRAM_NOALLOC_MAX_OWNERS 64

/* Return codes (0 = success; the message in `err` says more). */
#define ENGRAM_NOALLOC_BAD_SHAPE 1    /* layers or world outside the limits */
#define ENGRAM_NOALLOC_BAD_ROWS 2     /* tokens * ept beyond capacity or 32-bit indexing */
#define ENGRAM_NOALLOC_NULL_ARG 3     /* a required pointer is null */
#define ENGRAM_NOALLOC_NO_DEVICE 4    /* no current device, or the array's address lookup failed */
#define ENGRAM_NOALLOC_BAD_ENTRIES 5  /* an entries value is zero or the vocabulary exceeds the limits */
#define ENGRAM_NOALLOC_CUDA_ERROR 6   /* a CUDA call or the launch failed */

#ifdef __cplusplus
extern "C" {
#endif

/* entries_host: `layers` values; owners_host: `world` flags; err: a caller
 * buffer of err_len bytes for a NUL-terminated message (may be NULL). */
int engram_route_pack_noalloc(const int32_t *indices, uint32_t layers, uint32_t tokens, uint32_t ept,
                              const uint32_t *entries_host, uint32_t world, const uint8_t *owners_host,
                              int64_t *packed, uint32_t capacity, int32_t *counts, cudaStream_t stream, char *err,
                              size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* ENGRAM_NOALLOC_H */
