// extern "C" entry points to the normalisation / gate host launchers (norm.cu) of the emulated
// build; the test compiles this file after rewriting norm.cu for tests/csrc/host_emu.cuh.
#include "norm_emu_src.inc"

extern "C" {
int emu_error_word() { return ::emu::error_word.exchange(0); }

int emu_norm_grid(long long rows) { return maloq::norm_grid(rows); }

const char* emu_rms_norm_fwd(int L, const float* X, const float* RES, const float* aw, const float* ab, void* OUT,
                             int out_bf16, float* SUM, int B, int C, float eps) {
  return maloq::rms_norm_fwd(L, X, RES, aw, ab, OUT, out_bf16 != 0, SUM, B, C, eps, nullptr);
}

const char* emu_rms_norm_bwd(int L, const float* Sx, const void* G, int g_bf16, const float* GS, const float* aw,
                             float* DX, float* PART, int B, int C, float eps, int grid) {
  return maloq::rms_norm_bwd(L, Sx, G, g_bf16 != 0, GS, aw, DX, PART, B, C, eps, grid, nullptr);
}

const char* emu_ln_silu_fwd(const float* X, const float* w, const float* b, __nv_bfloat16* OUT, int M, int W, float eps) {
  return maloq::ln_silu_fwd(X, w, b, OUT, M, W, eps, nullptr);
}

const char* emu_ln_silu_bwd(const float* X, const float* w, const float* b, const __nv_bfloat16* G, float* DX,
                            float* PART, int M, int W, float eps, int grid) {
  return maloq::ln_silu_bwd(X, w, b, G, DX, PART, M, W, eps, grid, nullptr);
}

const char* emu_gate_l_fwd(int L, const void* X, const float* Gt, void* OUT, int bf16, int B, int H) {
  return maloq::gate_l_fwd(L, X, Gt, OUT, bf16 != 0, B, H, nullptr);
}

const char* emu_gate_l_bwd(int L, const void* X, const float* Gt, const void* DO, void* DX, float* DG, int bf16, int B,
                           int H) {
  return maloq::gate_l_bwd(L, X, Gt, DO, DX, DG, bf16 != 0, B, H, nullptr);
}

// the same with the gate pre-activation flag
const char* emu_gate_l_fwd_s(int L, const void* X, const float* Gt, void* OUT, int bf16, int B, int H, int silu_gates) {
  return maloq::gate_l_fwd(L, X, Gt, OUT, bf16 != 0, B, H, nullptr, silu_gates != 0);
}

const char* emu_gate_l_bwd_s(int L, const void* X, const float* Gt, const void* DO, void* DX, float* DG, int bf16,
                             int B, int H, int silu_gates) {
  return maloq::gate_l_bwd(L, X, Gt, DO, DX, DG, bf16 != 0, B, H, nullptr, silu_gates != 0);
}

const char* emu_head_gate_fwd(int L, const float* X, const float* SV, __nv_bfloat16* A, int act, float scale, int absg,
                              int B, int C) {
  return maloq::head_gate_fwd(L, X, SV, A, act, scale, absg != 0, B, C, nullptr);
}

const char* emu_head_gate_bwd(int L, const float* X, const float* SV, const float* DA, float* DX, float* DSV, int act,
                              float scale, int absg, int B, int C) {
  return maloq::head_gate_bwd(L, X, SV, DA, DX, DSV, act, scale, absg != 0, B, C, nullptr);
}
}
