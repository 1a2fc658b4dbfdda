// lb_gemm_bf16_noalloc: a split-K tensor-core GEMM entry point that allocates nothing.
//
// This entry point has no counterpart in the reference (ciresnave/lightbulb); it exists for
// callers of this library that cannot allocate device memory themselves: code running inside
// a custom allocator or memory-pool callback (where a nested cudaMalloc would recurse or
// deadlock), plugins hosted by a runtime that owns every device allocation (inference servers,
// frameworks with a fixed arena), and real-time paths where an allocation's latency or
// failure is not acceptable.  The caller passes device pointers to the inputs and the output
// only; the fp32 split-K partial tiles, the per-tile arrival counters and the error word live
// in one file-scope `static __device__` array inside the library.
//
//   C[M, N] (bf16) = A[M, K] (bf16, row stride lda) . W[N, K]^T (bf16, row stride ldw)
//
// Rules:
//  * Scratch limit: 16 MiB of partial tiles (4 Mi floats) and 16384 tiles.  A call whose
//    split-K plan needs more (tiles x splits x token_tile x 128 floats, token_tile = 16, 32,
//    64, 128 or 256 by M) is rejected with LB_NOALLOC_TOO_LARGE and a message on stderr;
//    nothing is launched.
//  * Every GPU that loads the library holds that array until the process exits.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress)
//    and sets the kernel's shared-memory attribute with that device current.  Make that first
//    call before any CUDA stream capture on the device.
//  * Every call shares the same array: calls that overlap on the GPU (different streams, or
//    different host threads, without ordering between them) race on it.  Calls ordered on one
//    stream are safe.  Each call clears the counters and error word it uses before its kernel.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
//
// Return value: 0 on success, otherwise one of the codes below (a message goes to stderr).
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LB_NOALLOC_OK = 0,
  LB_NOALLOC_BAD_ARGS = 1,    // null pointer, non-positive size, K % 8 != 0, misaligned rows
  LB_NOALLOC_TOO_LARGE = 2,   // split-K plan needs more scratch than the static maximum
  LB_NOALLOC_CUDA_ERROR = 3,  // a CUDA runtime/driver call failed (message on stderr)
};

// splits: number of K slices (>= 1); 1 = no partial tiles.
int lb_gemm_bf16_noalloc(const void* A, int lda, const void* W, int ldw, void* C, int ldc,
                         int M, int N, int K, int splits, cudaStream_t stream);

// Kernel-side status of the most recent lb_gemm_bf16_noalloc call on the current device.
// The GEMM kernel runs asynchronously, so a return of LB_NOALLOC_OK from the GEMM only means
// the launch was accepted.  Its bounded waits (TMA arrivals, tensor-core commits, split-K
// peers) record a nonzero code in the shared error word when they expire, in which case C is
// incomplete.  This function waits for `stream` (pass the stream of the GEMM), then stores
// that word in *kernel_error: 0 = the kernel finished normally; 1-7 = which wait expired
// (1 TMA full, 2 shared-memory empty, 3 TMEM full, 4 TMEM empty, 5 split-K peer, 6 bounds,
// 7 drain).  The word is cleared by the next GEMM call, so query it before issuing another.
// Allocates nothing.  Returns LB_NOALLOC_OK or LB_NOALLOC_CUDA_ERROR / LB_NOALLOC_BAD_ARGS.
int lb_gemm_bf16_noalloc_status(int* kernel_error, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
