// Host API of misc.cu.  Plain CUDA types.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace maloq {

const char* edge_rotation(const float* vec, long long ldv, const float* J, const int* joff, int L, const int* row_l,
                          const int* row_m, int R, float* ROT, int E, cudaStream_t st);
int fock_loss_grid(long long n);
// part: [grid, 3] = (sum of squared error, sum of absolute error, count) per CTA
const char* fock_loss_stats(const float* O, const float* Tt, const long long* pt, const uint8_t* mask, int D,
                            long long rows, float* part, int grid, long long n_pt, cudaStream_t st);
const char* fock_loss_grad(const float* O, const float* Tt, const long long* pt, const uint8_t* mask, int D,
                           long long rows, const float* gstat, float* G, long long n_pt, cudaStream_t st);

}  // namespace maloq
