// Allocation-free CRC-32 entry point.
//
// This entry point has no counterpart in the reference library; it exists for
// callers of this library that cannot allocate GPU memory at the moment they
// need a checksum:
//   * serving engines that reserve all free HBM for their own pool at start-up
//     (paged KV caches do this), so a later cudaMalloc fails or fragments
//     memory the pool owns;
//   * latency-critical paths, where cudaMalloc/cudaFree may synchronize the
//     device and stall every stream;
//   * plain C callers (through dlopen/ctypes) that have no CUDA allocator of
//     their own.
// The regular entry point (kern::crc32_blocks) grows a scratch buffer with
// cudaMalloc on demand; this one keeps its scratch in a fixed, file-scope
// __device__ array instead and allocates nothing.
//
// Scratch limit: MPCOMM_CRC32_NOALLOC_MAX_WORDS 32-bit words (256 KiB) per
// device, one word per 512 KiB piece of input, i.e. num_blocks *
// ceil(block_size / 512 KiB) <= 65536 (for example 4 blocks of 8 GiB, or
// 65536 blocks of up to 512 KiB). Larger requests are rejected with -1 and a
// message on stderr. Every GPU that loads the library holds the array until
// the process exits.
//
// Setup: the first call on each device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress; make that first call
// before any CUDA stream capture. The address is cached per device and
// context; a call in a context created since (after cudaDeviceReset, say)
// looks it up again, so that call too belongs outside a capture.
//
// Errors: a runtime error already pending when the call starts (left by the
// caller's earlier work) is returned as is, before anything is queued.
//
// Sharing: all calls on a device share the one array and it keeps the last
// call's contents. Each call writes every scratch word it later reads, in
// stream order, so nothing needs clearing between calls; but two calls that
// overlap on the GPU (different streams, no ordering between them) race on
// the array and may return wrong CRCs. Serialize them (same stream or events).
#ifndef MPCOMM_B200_CSRC_KERNELS_CRC32_NOALLOC_H_
#define MPCOMM_B200_CSRC_KERNELS_CRC32_NOALLOC_H_

#include <stdint.h>

#define MPCOMM_CRC32_NOALLOC_MAX_WORDS 65536

#ifdef __cplusplus
extern "C" {
#endif

// CRC-32 (zlib polynomial 0xEDB88320, init/final xor 0xFFFFFFFF) of
// num_blocks consecutive blocks of block_size bytes at device-accessible
// `data`, written to out[0..num_blocks) (device-accessible), launched on
// `stream` (a cudaStream_t; NULL = legacy default stream). Returns 0 on
// success, -1 if the request exceeds the scratch limit, otherwise the CUDA
// error code of the failed setup or launch.
__attribute__((visibility("default"))) int mpcomm_crc32_blocks_noalloc(
    const void *data, int64_t num_blocks, int64_t block_size, uint32_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif  // MPCOMM_B200_CSRC_KERNELS_CRC32_NOALLOC_H_
