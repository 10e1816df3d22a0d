// Fock-head gate kernels (included by norm.cu).
//
// Plain grid-stride kernels over (row, channel) with no shared memory, warp intrinsics or
// synchronisation, so this file also compiles as host C++: a test builds it with the host
// compiler, runs the kernels over an emulated grid on the CPU and compares them with PyTorch.
// That host build defines MALOQ_HOST_EMULATION and provides blockIdx / threadIdx / blockDim /
// gridDim.
#pragma once
#include <cuda_bf16.h>
#ifdef MALOQ_HOST_EMULATION
#include <cmath>
#endif

namespace maloq {

// SV [B, C + L*C] = (transformed scalars | raw gates), X [B, S, C] fp32.
// A[b,0,c] = SV[b,c]; A[b,j,c] = X[b,j,c] * scale * act(u), u = SV[b, C + (l_j-1)*C + c]
// (|u| with ABSG); act = sigmoid (ACT 0) or tanh (ACT 1).  A is the bf16 GEMM operand.
template <int ACT>
__device__ __forceinline__ float head_act(float u, float* dact) {
  if (ACT == 0) {
    const float a = 1.f / (1.f + expf(-u));
    *dact = a * (1.f - a);
    return a;
  }
  const float t = tanhf(u);
  *dact = 1.f - t * t;
  return t;
}

template <int L, int ACT>
__global__ void head_gate_fwd_kernel(const float* __restrict__ X, const float* __restrict__ SV,
                                     __nv_bfloat16* __restrict__ A, int B, int C, float scale, bool absg) {
  constexpr int S = (L + 1) * (L + 1);
  const long long total = (long long)B * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long b = i / C;
    const float* x = X + b * S * C + c;
    const float* sv = SV + b * (L + 1) * C + c;
    __nv_bfloat16* a = A + b * S * C + c;
    a[0] = __float2bfloat16_rn(sv[0]);
#pragma unroll
    for (int l = 1; l <= L; ++l) {
      const float u = sv[(size_t)l * C];
      float da;
      const float g = scale * head_act<ACT>(absg ? fabsf(u) : u, &da);
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) a[(size_t)j * C] = __float2bfloat16_rn(x[(size_t)j * C] * g);
    }
  }
}

// Backward from DA [B, S, C] fp32: DX[b,0,:] = 0 (row 0 of X does not enter A), DX[b,j,c] =
// DA * gate; DSV[b,c] = DA[b,0,c]; DSV of gate (l, c) = sum_j DA*X * scale * act'(u) (* sign(u)
// with ABSG, 0 at u = 0).
template <int L, int ACT>
__global__ void head_gate_bwd_kernel(const float* __restrict__ X, const float* __restrict__ SV,
                                     const float* __restrict__ DA, float* __restrict__ DX, float* __restrict__ DSV,
                                     int B, int C, float scale, bool absg) {
  constexpr int S = (L + 1) * (L + 1);
  const long long total = (long long)B * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long b = i / C;
    const float* x = X + b * S * C + c;
    const float* sv = SV + b * (L + 1) * C + c;
    const float* da = DA + b * S * C + c;
    float* dx = DX + b * S * C + c;
    float* dsv = DSV + b * (L + 1) * C + c;
    dx[0] = 0.f;
    dsv[0] = da[0];
#pragma unroll
    for (int l = 1; l <= L; ++l) {
      const float u = sv[(size_t)l * C];
      float dact;
      const float g = scale * head_act<ACT>(absg ? fabsf(u) : u, &dact);
      float acc = 0.f;
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
        const float d = da[(size_t)j * C];
        dx[(size_t)j * C] = d * g;
        acc += d * x[(size_t)j * C];
      }
      const float sgn = absg ? (u > 0.f ? 1.f : (u < 0.f ? -1.f : 0.f)) : 1.f;
      dsv[(size_t)l * C] = acc * scale * dact * sgn;
    }
  }
}


}  // namespace maloq
