// Host API of misc.cu.  Plain CUDA types.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace maloq {

const char* edge_rotation(const float* vec, long long ldv, const float* J, const int* joff, int L, const int* row_l,
                          const int* row_m, int R, float* ROT, int E, cudaStream_t st);
// Column sums out[N] (fp32) of X [M, N] (fp32, or bf16 when bf16) with row stride ld, in a fixed
// order.  P = colsum_chunks(M, N) row chunks; part: fp32 [P, N] scratch when P > 1 (else unused).
int colsum_chunks(long long M, int N);
const char* colsum(const void* X, bool bf16, long long M, int N, long long ld, float* part, int P, float* out,
                   cudaStream_t st);
// Segment sums out[s, N] = column sums of rows [seg[s], seg[s + 1]) of the fp32 X (row stride
// ld), s < nseg <= kColsumSegs; seg: host array of nseg + 1 non-decreasing row offsets.
constexpr int kColsumSegs = 32;
const char* colsum_segments(const float* X, int N, long long ld, const long long* seg, int nseg, float* out,
                            cudaStream_t st);
// Weight operand copies, job g: src fp32 [batch[g], rows[g], cols[g]] (contiguous) ->
//   kPackCast      dst bf16, same shape
//   kPackTranspose dst bf16 [batch, cols, rows]
//   kPackPair      dst bf16 [rows, 2 cols] = [[W_r, -W_i], [W_i, W_r]] of src = [W_r; W_i]
//   kPackPairT     dst bf16 [2 cols, rows], the transpose of the pair matrix
//   kPackPairGrad  dst fp32 [rows, cols / 2]: [dW_r; dW_i] from the pair matrix gradient src
// kPackJobs jobs per launch (the job table is a kernel parameter).
constexpr int kPackJobs = 48;
enum { kPackCast = 0, kPackTranspose = 1, kPackPair = 2, kPackPairT = 3, kPackPairGrad = 4 };
const char* weight_pack(int n, const float* const* src, void* const* dst, const int* batch, const int* rows,
                        const int* cols, const int* kind, cudaStream_t st);
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
