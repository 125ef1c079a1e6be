// Paged decode attention with built-in scratch: an entry point that allocates
// no device memory.
//
// This entry point has no counterpart in the reference. It exists for
// callers that cannot allocate at the moment they run attention:
//   * a host program that hands all of its device memory to a fixed pool at
//     start-up (weights plus the KV page pool) and must not grow afterwards,
//     so a stray cudaMalloc would either fail or steal from the KV pool;
//   * code that runs without PyTorch or any other caching allocator (a plain
//     C or C++ host linking only this library), which has no cheap place to
//     get a temporary buffer from and would otherwise pay a cudaMalloc and a
//     cudaFree, each of which synchronises the device, on every call;
//   * code that runs while an allocator is unavailable to it, for example
//     inside that allocator's own out-of-memory handling.
// Such callers use this function instead of b200_paged_decode, which takes
// its split-KV scratch (part_acc, part_ml) from the caller.
//
// Behaviour: the same two kernels as b200_paged_decode (the partition pass,
// then the merge pass) with the same arguments, except that the partial
// results live in a fixed array compiled into the library (a file-scope
// __device__ array of B200_DECODE_NOALLOC_SCRATCH_BYTES bytes, 8 MiB). The
// output is bit-identical to b200_paged_decode's.
//
// Size limit: the call needs
//     round_up(B * H * max_parts * D, 64) + B * H * max_parts * 2
// floats of scratch, which must not exceed B200_DECODE_NOALLOC_SCRATCH_FLOATS
// (2,097,152). Larger calls return B200_DECODE_NOALLOC_TOO_LARGE (-2) and
// launch nothing. Example: B = 64 rows, H = 32 heads, D = 128 fits up to
// max_parts = 7 (contexts up to 1792 tokens; a partition is 256 tokens).
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current, and keeps it for
// later calls on that device. That lookup may load the library's device code
// onto the device, so make the first call on each device before any stream
// capture begins. If the lookup fails, the call returns its CUDA error code
// and launches nothing.
//
// Nothing in the scratch has to start at zero: every partition slot that the
// merge pass reads is written by the partition pass of the same call.
//
// Concurrency: there is one scratch array per device. Two calls whose kernels
// can run at the same time on one device (calls on different streams without
// an ordering between them, or from several host threads onto different
// streams) race on it and produce wrong results. Calls issued in order on
// one stream are safe.
//
// Returns 0 on success, -1 for an unsupported shape (D not 64/128/256, H not
// a multiple of KVH, or an unsupported group size), -2 when the scratch
// would exceed the limit, or a CUDA error code.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define B200_DECODE_NOALLOC_SCRATCH_FLOATS (2 * 1024 * 1024)
#define B200_DECODE_NOALLOC_SCRATCH_BYTES (B200_DECODE_NOALLOC_SCRATCH_FLOATS * 4)
#define B200_DECODE_NOALLOC_TOO_LARGE (-2)

#ifdef __cplusplus
extern "C" {
#endif

int b200_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, int kv_fp8,
                              const float* k_scale, const float* v_scale, const int* page_table, int ld_pt,
                              const int* seq_lens, const float* sinks, void* out, int B, int H, int KVH, int D,
                              int max_parts, int window, float scale, float softcap, int64_t num_pages,
                              cudaStream_t st);

#ifdef __cplusplus
}
#endif
