// Host API of norm.cu.  Plain CUDA types.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace maloq {

int norm_grid(long long rows);
// OUT: fp32, or bf16 when out_bf16 (an output that only feeds a bf16 GEMM)
const char* rms_norm_fwd(int L, const float* X, const float* RES, const float* aw, const float* ab, void* OUT,
                         bool out_bf16, float* SUM, int B, int C, float eps, cudaStream_t st);
// G: gradient of OUT (fp32, or bf16 when g_bf16).  PART: [grid, L+2, C] partial
// (d_affine_weight, d_affine_bias) per CTA
const char* rms_norm_bwd(int L, const float* Sx, const void* G, bool g_bf16, const float* GS, const float* aw,
                         float* DX, float* PART, int B, int C, float eps, int grid, cudaStream_t st);
const char* ln_silu_fwd(const float* X, const float* w, const float* b, __nv_bfloat16* OUT, int M, int W, float eps,
                        cudaStream_t st);
// PART: [grid * 8, 2, W] partial (d_weight, d_bias) per warp (256-thread CTAs)
const char* ln_silu_bwd(const float* X, const float* w, const float* b, const __nv_bfloat16* G, float* DX, float* PART,
                        int M, int W, float eps, int grid, cudaStream_t st);
// X / OUT / DO / DX: fp32, or bf16 when bf16; gates Gt and their gradient DG fp32
// silu_gates: Gt holds pre-activations g, the gate is tanh(silu(g)) and DG is the gradient wrt g
const char* gate_l_fwd(int L, const void* X, const float* Gt, void* OUT, bool bf16, int B, int H, cudaStream_t st,
                       bool silu_gates = false);
const char* gate_l_bwd(int L, const void* X, const float* Gt, const void* DO, void* DX, float* DG, bool bf16, int B,
                       int H, cudaStream_t st, bool silu_gates = false);
// Fock-head gate: X [B, (L+1)^2, C] fp32, SV [B, (L+1) C] fp32 (transformed scalars | raw
// gates), A [B, (L+1)^2, C] bf16; act 0 sigmoid, 1 tanh; gates = scale * act(|u| if absg else u).
// Backward: DA fp32 -> DX (row 0 zero), DSV.
const char* head_gate_fwd(int L, const float* X, const float* SV, __nv_bfloat16* A, int act, float scale, bool absg,
                          int B, int C, cudaStream_t st);
const char* head_gate_bwd(int L, const float* X, const float* SV, const float* DA, float* DX, float* DSV, int act,
                          float scale, bool absg, int B, int C, cudaStream_t st);

}  // namespace maloq
