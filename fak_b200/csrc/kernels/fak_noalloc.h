// fak_noalloc.h -- C declaration of the allocation-free decode attention entry point.
//
// This entry point has no counterpart in the reference; it is an addition of this library.
//
// Who it is for: callers that cannot allocate device memory while they run.  A C or C++ host
// runtime (or Python through ctypes) that links this library without PyTorch has no caching
// allocator to lend it a split-KV workspace, and a cudaMalloc/cudaFree pair per call would cost
// more than the kernel itself -- cudaFree also waits for the whole device.  A server that sizes
// its memory once at start-up (the KV page pool takes nearly all of HBM) likewise wants no
// allocation inside its decode loop, where an out-of-memory error would surface long after the
// request was admitted.  So this variant keeps its split-KV partial results in one statically
// sized device array (a file-scope __device__ array of attention.cu) and calls no allocator:
// no cudaMalloc, no cudaFree, no torch tensor.  The caller still passes every input and output.
//
// Limits: B * H * n_split <= FAK_NOALLOC_MAX_SLOTS (sequence, head, split) slots, head_dim 64 or 128
// (the array holds FAK_NOALLOC_MAX_SLOTS * (128 + 2) floats = 2,129,920 bytes on every device that
// loads the library, until the process exits).  A larger call returns FAK_NOALLOC_ETOOBIG and launches
// nothing.  n_split == 1 uses no scratch and has no size limit.
//
// Set-up: the first call that needs the scratch on a device (that device current) looks the array's
// device address up with cudaGetSymbolAddress and caches it for that device.  Make that first call
// before any stream capture begins.  The cached address belongs to the device's primary context:
// do not call cudaDeviceReset (or otherwise reset the primary context) between calls in a process
// that uses this entry point.
//
// Concurrency: every call on a device shares the one array, and the array keeps the last call's
// contents.  Nothing in it needs to start at zero (the attention kernel writes every slot, empty
// splits included, before the merge kernel reads it).  Two calls that overlap on the GPU (different
// streams, or host threads without ordering) race on the array and corrupt each other's results:
// issue them on one stream or order them yourself.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FAK_NOALLOC_MAX_SLOTS 4096
#define FAK_NOALLOC_OK 0
#define FAK_NOALLOC_EINVAL 1   /* invalid argument: nothing launched */
#define FAK_NOALLOC_ETOOBIG 2  /* B * H * n_split beyond FAK_NOALLOC_MAX_SLOTS: nothing launched */
#define FAK_NOALLOC_ECUDA 3    /* a CUDA runtime call failed */

// Split-KV paged decode attention for B sequences over a 16-token-page bf16 KV cache.
//   q            [B, H, D] f32 device, contiguous (queries after RoPE)
//   k_cache      [pages, Hkv, 16, D] bf16 device; v_cache the same
//   block_table  [B, bt_stride] int32 device: physical page of each sequence's 16-token page
//   ctx_len      [B] int32 device: keys attended per sequence (>= 1)
//   n_split      context splits per (sequence, KV head); pages_per_split is a lower bound on the pages
//                one split takes -- the kernel raises it to ceil(live pages / n_split), so every key is
//                attended whatever the value (pass 1 for an even spread)
//   out          [B, ldo] f32 device or NULL; qx [B, ldo] int8 + ds [B, ldo / 32, 2] f32 device or NULL:
//                at least one of out / qx; ds is required with qx (int8 codes and per-32 (scale, sum))
//   ldo          elements per output row (0 = H * D; otherwise >= H * D and a multiple of 32)
//   stream       cudaStream_t to launch on (NULL = the legacy default stream)
//   err, err_len optional buffer for a message on failure
// Returns FAK_NOALLOC_OK or one of the error codes above.
int fak_decode_attention_noalloc(const float* q, const void* k_cache, const void* v_cache, const int* block_table,
                                 int bt_stride, const int* ctx_len, int B, int H, int Hkv, int D, int n_split,
                                 int pages_per_split, float* out, int8_t* qx, float* ds, int ldo, void* stream,
                                 char* err, size_t err_len);

#ifdef __cplusplus
}
#endif
