// Allocation-free C entry point for decode attention.
//
// This entry point has no counterpart in the reference (which has no attention or
// model code at all); it is an addition of this library.
//
// Who it is for: callers that cannot allocate device memory at the moment they run
// attention: inference engines that reserve nearly all of the GPU's memory up front for
// their own pool (a stray cudaMalloc there can fail or fragment the pool), and plain
// C/C++ hosts that have no caching allocator and cannot afford cudaMalloc's implicit
// device synchronisation on a latency-critical path.
// Such callers pass only their inputs and output; the per-split partial results the
// kernels need live in a fixed scratch array compiled into the library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Bytes of the library's built-in attention scratch (held by every GPU that loads the
// library, until the process exits).
#define SPARKNET_NOALLOC_SCRATCH_BYTES (8u << 20)

// Decode attention, one query token per sequence, head_dim 128, bf16:
//   q        [B, Hq, 128]            k_cache, v_cache [B, Lmax, Hkv, 128]
//   lengths  [B] int32 (keys to attend, including the new token)
//   out      [B, Hq, 128]            (all device pointers)
//   max_len  upper bound of lengths (decides the split of each sequence).  A length
//            above max_len is not an error and is not detected: such a sequence is
//            attended over its first max_len keys (rounded up to the split size) only,
//            which gives a wrong output for it.
//   scale    softmax scale (usually 1/sqrt(128))
// Returns 0 on success, or a nonzero code with a message from
// sparknet_noalloc_last_error(): 1 bad argument, 2 problem too large for the built-in
// scratch, 3 CUDA error.  Clears the call's counters and launches one kernel, both on
// `stream`; allocates nothing.
//
// The first call on a device looks up the device address of the scratch array (a
// CUDA runtime query, done once per device with that device current; concurrent first
// calls from several host threads are safe); make that first call outside any stream
// capture.  The address is cached for the life of the process: after a
// cudaDeviceReset of a device, do not call this entry point on that device again.  Every call, on every stream, shares the
// one scratch array, so calls that may overlap on the GPU (different streams, no
// ordering between them) race and must not be issued.  The scratch keeps the last
// call's contents.  It starts with a fixed block of per-(sequence, KV head) counters
// that must be zero when the kernel starts: each call zeroes the B x Hkv counters it
// uses (cudaMemsetAsync on `stream`, before its kernel), so nothing depends on how an
// earlier call ended.  The partials after them are written before they are read in
// every call.
__attribute__((visibility("default"))) int sparknet_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* lengths, void* out, int B, int Hq,
    int Hkv, int Lmax, int max_len, float scale, cudaStream_t stream);

// The message of the last failed call on this host thread ("" after a success).
__attribute__((visibility("default"))) const char* sparknet_noalloc_last_error(void);

// Bytes of scratch a problem needs on the current device (its SM count decides the
// split), 0 if the arguments are invalid or no device is current; compare with
// SPARKNET_NOALLOC_SCRATCH_BYTES.
__attribute__((visibility("default"))) size_t sparknet_decode_attention_scratch_bytes(int B, int Hq, int Hkv,
                                                                                       int max_len);

#ifdef __cplusplus
}
#endif
