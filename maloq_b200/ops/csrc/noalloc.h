// Allocation-free weight-gradient GEMM: exported C entry points (defined in noalloc.cu).
//
// These entry points have no counterpart in the reference.  They serve callers that cannot
// call cudaMalloc (or any allocator) from the code that launches the work: a host
// application that hands this library fixed buffers it allocated up front, a runtime that
// forbids allocation inside its step function, or code running while a memory pool is
// frozen.  The caller passes inputs and output; the split-K partial sums, which the regular
// path keeps in a freshly allocated workspace, live in one fixed device array here.
//
// Limits:
// * the array holds MALOQ_NOALLOC_SCRATCH_FLOATS fp32 values (64 MiB) and is held by every
//   GPU that loads the library until the process exits;
// * N*K must satisfy 2*N*K <= MALOQ_NOALLOC_SCRATCH_FLOATS (room for two split-K slices);
//   larger N*K is rejected with an error.  Calls whose M is too small for split-K (under
//   2048 rows) write dW directly and leave the array untouched;
// * every call shares the one array, so calls whose GPU work overlaps (two streams at once)
//   race on it: issue them in order on one stream or synchronise between them;
// * the first call on a device looks up the array's device address (cudaGetSymbolAddress,
//   with that device current) and caches it: make that first call before any stream capture.
#pragma once
#include <cuda_runtime.h>

#define MALOQ_NOALLOC_SCRATCH_FLOATS (16ll * 1024 * 1024)

#ifdef __cplusplus
extern "C" {
#endif

// dW[N,K] = gy[M,N]^T x[M,K] on `stream` without allocating.  gy and x are row-major bf16
// (16-byte aligned, N and K multiples of 8); dW is row-major fp32 [N,K].  Returns 0 on
// success, 1 on a rejected call (text from maloq_noalloc_last_error).
int maloq_weight_grad_noalloc(const void* gy, const void* x, float* dw, int M, int N, int K, cudaStream_t stream);

// Text of the last error returned by maloq_weight_grad_noalloc (nullptr if none).
const char* maloq_noalloc_last_error(void);

// Scratch capacity in fp32 elements (MALOQ_NOALLOC_SCRATCH_FLOATS).
long long maloq_noalloc_scratch_floats(void);

#ifdef __cplusplus
}
#endif
