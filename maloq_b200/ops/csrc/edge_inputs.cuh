// Radial-MLP input rows of every edge in one pass (included by misc.cu).
//
// OUT[e] = [ SRC_TABLE[src_z[e]] | exp(coeff (d_e - offset_k)^2), k < NB | DST_TABLE[dst_z[e]] ]
// (C + NB + C bf16 values): the element embeddings of the edge's source and target atoms around
// the Gaussian expansion of its length (reference helm/esen_osh.py:401-411 and
// helm/nn/radial.py:44-60 build the same row from three tensors and a concatenation).
//
// A plain grid-stride kernel over (edge, column) without shared memory or synchronisation, so
// this file also compiles as host C++: a test builds it with the host compiler, runs it over an
// emulated grid on the CPU and compares it with PyTorch (the host build defines
// MALOQ_HOST_EMULATION and provides blockIdx / threadIdx / blockDim / gridDim; a build through the
// test runtime, which defines MALOQ_EMU_RUNTIME, brings its own error word).
#pragma once
#include <cuda_bf16.h>
#if defined(MALOQ_HOST_EMULATION) && !defined(MALOQ_EMU_RUNTIME)
#include <cmath>
namespace maloq {
constexpr int ERR_BOUNDS = 5;
inline int g_emulated_error = 0;
inline void record_error(int code) {
  if (g_emulated_error == 0) g_emulated_error = code;
}
}  // namespace maloq
#endif

namespace maloq {

// D: edge lengths with stride ld_d; tables [n_types, C] fp32; an element index outside the
// table writes zeros and records ERR_BOUNDS in the device error word.
__global__ void edge_inputs_kernel(const long long* __restrict__ src_z, const long long* __restrict__ dst_z,
                                   const float* __restrict__ D, long long ld_d, const float* __restrict__ src_table,
                                   const float* __restrict__ dst_table, long long n_types,
                                   const float* __restrict__ offset, float coeff, __nv_bfloat16* __restrict__ OUT,
                                   long long E, int C, int NB) {
  const int W = 2 * C + NB;
  const long long total = E * W;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i / W;
    const int col = (int)(i - e * W);
    float v = 0.f;
    if (col < C || col >= C + NB) {
      const bool src = col < C;
      const long long t = src ? src_z[e] : dst_z[e];
      if (t >= 0 && t < n_types) {
        v = src ? src_table[t * C + col] : dst_table[t * C + (col - C - NB)];
      } else {
        record_error(ERR_BOUNDS);
      }
    } else {
      const float x = D[e * ld_d] - offset[col - C];
      v = expf(coeff * x * x);
    }
    OUT[i] = __float2bfloat16_rn(v);
  }
}

}  // namespace maloq
