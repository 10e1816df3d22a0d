// Host API of misc.cu.  Plain CUDA types.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
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
// Radial-MLP inputs OUT [E, 2C + NB] bf16 = [src_table[src_z] | gaussians of D | dst_table[dst_z]]
const char* edge_inputs(const long long* src_z, const long long* dst_z, const float* D, long long ld_d,
                        const float* src_table, const float* dst_table, long long n_types, const float* offset,
                        float coeff, __nv_bfloat16* OUT, long long E, int C, int NB, cudaStream_t st);

}  // namespace maloq
