// Host API of the edge-frame kernels (edge.cu).  Plain CUDA types.  L = lmax, MM = mmax.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace maloq {

// peers/halo_owner/halo_row/n_own: optional halo (source rows >= n_own read from peers'
// staging buffers); pass peers = nullptr when every source row is local.
// rad / DRAD: radial modulation [E, NS*Cin] bf16 (nullptr: no modulation).
const char* edge_gather_rotate_fwd(int L, int MM, const float* X, const float* XE, const long long* src,
                                   const long long* dst, const float* rot, const __nv_bfloat16* rad,
                                   __nv_bfloat16* A, int E, int C, int Cin, const float* const* peers,
                                   const int* halo_owner, const long long* halo_row, long long n_own,
                                   long long n_x_rows, long long n_halo, cudaStream_t st);
// Backward: DX [N, S, C] (N rows of the source space, written completely - or, with recv, the
// halo rows stored into their owners' receive slots instead), DXE (Cin = 3C), DRAD.  dst_ptr
// has N+1 entries (rows without incoming edges have empty ranges).
const char* edge_gather_rotate_bwd(int L, int MM, const float* X, const float* XE, const float* rot,
                                   const __nv_bfloat16* rad, const __nv_bfloat16* dA, const long long* dst_ptr,
                                   const long long* src_perm, const long long* src_ptr, float* DX, float* DXE,
                                   __nv_bfloat16* DRAD, int N, int E, int C, int Cin, const float* const* peers,
                                   const int* halo_owner, const long long* halo_row, long long n_own,
                                   long long n_x_rows, long long n_halo, cudaStream_t st,
                                   float* const* recv = nullptr, const long long* recv_slot = nullptr);
const char* edge_halo_fetch(const float* const* peers, const int* halo_owner, const long long* halo_row, float* out,
                            long long n_halo, int SC, cudaStream_t st);
const char* edge_halo_push(const float* G, float* const* recv, const int* halo_owner, const long long* recv_slot,
                           long long n_halo, int SC, cudaStream_t st);
const char* edge_node_reduce(const float* DDST, const long long* dst_ptr, const float* DSRC, const long long* src_perm,
                             const long long* src_ptr, float* DX, int N, int SC, long long n_dst_rows,
                             long long n_src_rows, cudaStream_t st);
const char* edge_rotate_back_scatter(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot,
                                     const long long* dst_ptr, const float* base, float* out, int N, int C, int Rk,
                                     float scale, cudaStream_t st);
const char* edge_rotate_back(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot, float* out,
                             int E, int C, int Rk, cudaStream_t st);
const char* edge_rotate_grad(int L, int MM, const float* G, const long long* rows, const float* rot,
                             __nv_bfloat16* DY, float* DYf, int E, int C, int Rk, float scale, cudaStream_t st);
const char* edge_gate_fwd(int L, int MM, const __nv_bfloat16* Y1, __nv_bfloat16* H1, int E, int H, cudaStream_t st);
const char* edge_gate_bwd(int L, int MM, const __nv_bfloat16* Y1, const __nv_bfloat16* dH1, __nv_bfloat16* dY1, int E,
                          int H, cudaStream_t st);

}  // namespace maloq
