// Allocation-free weight-gradient GEMM (declared in noalloc.h, which states the callers it
// serves and its limits; no counterpart in the reference).
//
//   dW[N,K] = gy[M,N]^T @ x[M,K]      (bf16 inputs, fp32 output and accumulation)
//
// The number of split-K slices follows the allocating path (gemm_tn_weight_grad in
// ops/kernels.py): min(ceil(296 / output tiles), M / 1024, 64).  When that is below two the
// GEMM writes dW directly and the scratch array is not touched.  Otherwise the partials go to
// the scratch array (as many slices as fit) and a fixed-order reduction writes dW; every
// partial element a reduction reads is written by the GEMM of the same call first, so nothing
// needs clearing between calls.  No cudaMalloc, cudaFree or allocating library routine is
// called.
#include "common.cuh"
#include "gemm.h"
#include "noalloc.h"

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

const char* maloq_noalloc_last_error(void) { return g_noalloc_error; }

long long maloq_noalloc_scratch_floats(void) { return MALOQ_NOALLOC_SCRATCH_FLOATS; }

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
  if (splits * slice > MALOQ_NOALLOC_SCRATCH_FLOATS) splits = MALOQ_NOALLOC_SCRATCH_FLOATS / slice;
  if (splits < 2) {
    // one slice: the GEMM writes dW itself
    maloq::GemmProblem p;
    p.a = gy;
    p.lda = N;
    p.b = x;
    p.ldb = K;
    p.c = dw;
    p.ldc = K;
    p.split_stride = slice;
    p.bias = nullptr;
    p.M = N;
    p.N = K;
    p.K = M;
    const char* err = maloq::gemm_launch(&p, 1, true, true, true, 0, 1.f, 1, 128, stream);
    return err ? fail(err) : 0;
  }
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
