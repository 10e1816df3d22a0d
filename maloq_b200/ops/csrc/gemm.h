// Host API of the tcgen05 GEMM (gemm.cu).  Plain CUDA types, no torch.
#pragma once
#include <cuda_runtime.h>

namespace maloq {

struct GemmProblem {
  const void* a;       // bf16, row-major; [M,K] (K-major) or [K,M] (MN-major)
  long long lda;       // row stride of a, elements
  const void* b;       // bf16, row-major; [N,K] or [K,N]
  long long ldb;
  void* c;             // row-major [M,N] (or [splits][M][N] for split-K), fp32 or bf16
  long long ldc;
  long long split_stride;  // elements between split-K outputs
  const float* bias;   // [N] or nullptr
  const float* resid = nullptr;  // fp32 [M, N] rows added in the epilogue (row stride ldr), or nullptr
  long long ldr = 0;
  int M, N, K;
};

// Launch up to eight problems in one kernel.  Returns an error string or nullptr.
const char* gemm_launch(const GemmProblem* probs, int nprob, bool a_mn, bool b_mn, bool out_fp32, int act,
                        float alpha, int splits, int bn, cudaStream_t stream);

const char* gemm_splitk_reduce(const float* part, float* out, long long n, int splits, long long stride, float beta,
                               cudaStream_t stream);

}  // namespace maloq
