// Allocation-free C entry point for the split-K sparse MLA decode.
//
// This entry point has no counterpart in the reference project; it exists for
// hosts that embed these kernels but must not allocate device memory while
// serving.  Examples: an inference runtime that reserves all HBM up front and
// hands kernels only pre-planned buffers, a process whose device allocator is
// owned by another framework, or a latency-critical loop where a cudaMalloc
// (and the implicit synchronisation it can cause) is not allowed.  The regular
// Python/torch entry point gets its split-K scratch from the torch caching
// allocator; this one instead uses a fixed scratch array compiled into the
// library, so the caller passes only inputs and outputs.
//
// Scratch: a file-scope device array sized for splits * T <= CXLD_NOALLOC_MLA_MAX_ROWS
// (128 heads x (512 + 1) FP32 per row, about 8.4 MB).  Every GPU that loads the
// library holds this array until the process exits.
//
// Behaviour the caller must know:
//  * The first call on a device (with that device current) resolves the
//    array's device address with cudaGetSymbolAddress; make that first call
//    before any stream capture on that device.
//  * All calls share the one array and it keeps the previous call's contents
//    (every split overwrites its own partial rows, so nothing needs clearing).
//    Calls that overlap on the GPU (different streams, no ordering between
//    them) race on the array and produce wrong results; serialise them.
//  * Requests with splits * T above the maximum are rejected with
//    CXLD_NOALLOC_TOO_LARGE and nothing is launched.
//  * Device-side failures (a bounded wait that ran out, for instance) do not
//    change the return code, which only covers argument checks and the
//    launch.  The kernel records them in a device error word of the library
//    that each call clears, in stream order, before its kernel runs; read it
//    with cxld_sparse_mla_noalloc_error after the call (0 = no error, else a
//    device error code).  The word is shared like the scratch array.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#pragma once
#include <cuda_runtime.h>

#define CXLD_NOALLOC_MLA_MAX_ROWS 32

#define CXLD_NOALLOC_OK 0
#define CXLD_NOALLOC_BAD_ARGUMENT 1
#define CXLD_NOALLOC_TOO_LARGE 2
#define CXLD_NOALLOC_SETUP_FAILED 3
#define CXLD_NOALLOC_LAUNCH_FAILED 4

#ifdef __cplusplus
extern "C" {
#endif

// out[t, h, :] = sparse MLA of q[t] over kv rows ids[t, :K] (padding: -1 or >= P),
// split over `splits` key ranges and merged with a log-sum-exp combine.
// q: BF16 [T, 128, 576]; kv: BF16 [P, 576]; ids: int32 [T, K]; out: BF16
// [T, 128, 512]; lse: FP32 [T, 128] (natural log) or NULL.  All pointers are
// device pointers; work is enqueued on `stream`.  Returns a CXLD_NOALLOC_* code.
__attribute__((visibility("default"))) int cxld_sparse_mla_split_noalloc(
    const void* q, const void* kv, const int* ids, int T, int K, int P, float scale, int splits,
    void* out, float* lse, cudaStream_t stream);

// Device error code of the most recent call on `stream`'s device: waits for
// the work already enqueued on `stream`, then stores the code in
// *device_code (0 when the call's kernels recorded no error).  Returns a
// CXLD_NOALLOC_* code for the read itself.
__attribute__((visibility("default"))) int cxld_sparse_mla_noalloc_error(int* device_code, cudaStream_t stream);

// Largest splits * T a call accepts.
__attribute__((visibility("default"))) int cxld_sparse_mla_noalloc_max_rows(void);

// Human-readable text of a CXLD_NOALLOC_* code.
__attribute__((visibility("default"))) const char* cxld_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
