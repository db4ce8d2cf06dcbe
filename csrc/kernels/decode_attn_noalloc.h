// Allocation-free split-KV decode attention: C declarations.
//
// This entry point has no counterpart in the reference. It is for callers that cannot
// allocate GPU memory at call time (a host framework that owns the device memory
// budget, a plugin of another runtime that only hands over input and output buffers):
// its split-KV scratch is one fixed device array compiled into the library,
// AXR_NOALLOC_SCRATCH_FLOATS fp32 values (8 MiB) per GPU, held until the process exits.
//
// Rules for callers:
//  * One call needs B * Hq * num_splits * (head_dim + 1) floats of scratch (none with
//    num_splits == 1); larger calls return AXR_NOALLOC_TOO_LARGE and launch nothing.
//  * Every call on a device shares the one array. Calls that overlap on the GPU (two
//    streams, or two threads launching at once) race on it: serialise them.
//  * The first call on each device resolves the array's device address
//    (cudaGetSymbolAddress) with that device current. Make it before any stream
//    capture.
//  * block_table rows hold bt_stride entries; max_pages <= bt_stride. Pages at or past
//    max_pages are never read, so seq_lens[b] <= max_pages * 16 must hold for the
//    result to cover the whole sequence (a longer sequence is cut at max_pages * 16).
//  * The call never allocates or frees device memory and never calls an allocating
//    library routine.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AXR_NOALLOC_SCRATCH_FLOATS 2097152LL

enum AxrNoAllocStatus {
  AXR_NOALLOC_OK = 0,
  AXR_NOALLOC_TOO_LARGE = 1,      // the call needs more scratch than the fixed array
  AXR_NOALLOC_SETUP_FAILED = 2,   // the per-device address lookup failed
  AXR_NOALLOC_BAD_ARGS = 3,       // null pointers, unsupported shape, max_pages > bt_stride, ...
  AXR_NOALLOC_LAUNCH_FAILED = 4,  // a kernel launch of this call returned an error
  AXR_NOALLOC_PENDING_ERROR = 5,  // an earlier, unrelated CUDA error was pending; left in place, nothing launched
};

// Largest number of fp32 scratch elements one call may use.
long long axr_decode_noalloc_scratch_floats(void);

// Reason of this thread's last non-zero return (static string, never freed).
const char* axr_decode_noalloc_last_error(void);

// q, out: bf16 [B, Hq, D]; k_pages / v_pages: bf16 pages [block][head][16][D] of one
// layer (blk_stride / head_stride in bytes); block_table int32 [B, bt_stride];
// seq_lens int32 [B]. D = 128, Hq / Hkv in {1, 2, 4, 8}.
int axr_decode_attention_noalloc(const void* q, void* out, const void* k_pages, const void* v_pages,
                                 long long blk_stride, long long head_stride, const int* block_table, int bt_stride,
                                 const int* seq_lens, int B, int Hq, int Hkv, int D, float scale, int num_splits,
                                 int max_pages, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
