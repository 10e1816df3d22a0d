// Allocation-free weight-gradient GEMM: a C entry point for callers that cannot allocate.
//
// This entry point has no counterpart in the reference.  It exists for callers that must
// not call cudaMalloc (or any allocator) from the code that launches the work: a host
// application that hands this library fixed buffers it allocated up front, a runtime that
// forbids allocation inside its step function, or code running while a memory pool is
// frozen.  Such callers pass the inputs and the output; the split-K partial sums that the
// regular path (gemm_tn_weight_grad in ops/kernels.py) keeps in a freshly allocated
// workspace live here in a fixed-size device array instead.
//
//   dW[N,K] = gy[M,N]^T @ x[M,K]      (bf16 inputs, fp32 output and accumulation)
//
// Limits and behaviour:
// * The scratch array holds MALOQ_NOALLOC_SCRATCH_FLOATS fp32 values (64 MiB).  Every GPU
//   that loads this library reserves it until the process exits.  The call uses
//   s = min(desired splits, scratch / (N*K)) partial slices and is rejected with an error
//   when even two slices (2*N*K floats) do not fit.
// * The first call on each device looks up the array's device address with
//   cudaGetSymbolAddress (with that device current) and caches it; make that first call
//   before any stream capture.
// * All calls share the one array and each call overwrites the slices it uses (every
//   partial element is written before it is read, so nothing needs clearing).  Calls whose
//   GPU work overlaps - on two streams at once, for example - race on the array; issue them
//   in order on one stream or synchronise between them.
// * No cudaMalloc, cudaFree or allocating library routine is called.
#include "common.cuh"
#include "gemm.h"

#define MALOQ_NOALLOC_SCRATCH_FLOATS (16ll * 1024 * 1024)
#define MALOQ_NOALLOC_MAX_DEVICES 64

namespace {

static __device__ __align__(256) float g_noalloc_scratch[MALOQ_NOALLOC_SCRATCH_FLOATS];

float* g_noalloc_ptr[MALOQ_NOALLOC_MAX_DEVICES] = {nullptr};
const char* g_noalloc_error = nullptr;

int fail(const char* msg) {
  g_noalloc_error = msg;
  return 1;
}

}  // namespace

extern "C" {

// Text of the last error returned by maloq_weight_grad_noalloc (nullptr if none).
const char* maloq_noalloc_last_error() { return g_noalloc_error; }

// Scratch capacity in fp32 elements.
long long maloq_noalloc_scratch_floats() { return MALOQ_NOALLOC_SCRATCH_FLOATS; }

// dW[N,K] = gy[M,N]^T x[M,K] on `stream` without allocating.  gy and x are row-major bf16
// (16-byte aligned, N and K multiples of 8); dW is row-major fp32 [N,K].  Returns 0 on
// success, 1 on a rejected call (see maloq_noalloc_last_error).
int maloq_weight_grad_noalloc(const void* gy, const void* x, float* dw, int M, int N, int K, cudaStream_t stream) {
  g_noalloc_error = nullptr;
  if (M < 0 || N <= 0 || K <= 0) return fail("maloq_weight_grad_noalloc: bad sizes");
  if (N % 8 != 0 || K % 8 != 0) return fail("maloq_weight_grad_noalloc: N and K must be multiples of 8");
  const long long slice = (long long)N * K;
  if (2 * slice > MALOQ_NOALLOC_SCRATCH_FLOATS)
    return fail("maloq_weight_grad_noalloc: N*K too large for the 64 MiB scratch array (need 2*N*K <= 16M floats)");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MALOQ_NOALLOC_MAX_DEVICES)
    return fail("maloq_weight_grad_noalloc: no usable current device");
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return fail("maloq_weight_grad_noalloc: cudaGetSymbolAddress of the scratch array failed");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  float* scratch = g_noalloc_ptr[dev];
  if (M == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * slice, stream);
    return e == cudaSuccess ? 0 : fail("maloq_weight_grad_noalloc: cudaMemsetAsync failed");
  }
  const int tiles = ((N + 127) / 128) * ((K + 127) / 128);
  long long splits = (296 + tiles - 1) / tiles;
  if (splits > M / 1024) splits = M / 1024;
  if (splits > 64) splits = 64;
  if (splits < 2) splits = 2;
  if (splits * slice > MALOQ_NOALLOC_SCRATCH_FLOATS) splits = MALOQ_NOALLOC_SCRATCH_FLOATS / slice;
  maloq::GemmProblem p;
  p.a = gy;
  p.lda = N;
  p.b = x;
  p.ldb = K;
  p.c = scratch;
  p.ldc = K;
  p.split_stride = slice;
  p.bias = nullptr;
  p.M = N;
  p.N = K;
  p.K = M;
  const char* err = maloq::gemm_launch(&p, 1, true, true, true, 0, 1.f, (int)splits, 128, stream);
  if (err) return fail(err);
  err = maloq::gemm_splitk_reduce(scratch, dw, slice, (int)splits, slice, 0.f, stream);
  if (err) return fail(err);
  return 0;
}

}  // extern "C"
