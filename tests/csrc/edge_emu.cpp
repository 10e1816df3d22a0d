// extern "C" entry points to the edge-frame host launchers (edge.cu) of the emulated build; the
// test compiles this file after rewriting edge.cu for tests/csrc/host_emu.cuh.
#include "edge_emu_src.inc"

extern "C" {
int emu_error_word() { return ::emu::error_word.exchange(0); }

const char* emu_gather_rotate_fwd(int L, int MM, const float* X, const float* XE, const long long* src,
                                  const long long* dst, const float* rot, const __nv_bfloat16* rad, __nv_bfloat16* A,
                                  int E, int C, int Cin, long long n_x_rows) {
  return maloq::edge_gather_rotate_fwd(L, MM, X, XE, src, dst, rot, rad, A, E, C, Cin, nullptr, nullptr, nullptr, 0,
                                       n_x_rows, 0, nullptr);
}

const char* emu_gather_rotate_bwd(int L, int MM, const float* X, const float* XE, const float* rot,
                                  const __nv_bfloat16* rad, const __nv_bfloat16* dA, const long long* dst_ptr,
                                  const long long* src_perm, const long long* src_ptr, float* DX, float* DXE,
                                  __nv_bfloat16* DRAD, int N, int E, int C, int Cin) {
  return maloq::edge_gather_rotate_bwd(L, MM, X, XE, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DXE, DRAD, N, E, C,
                                       Cin, nullptr, nullptr, nullptr, 0, N, 0, nullptr);
}

const char* emu_rotate_back_scatter(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot,
                                    const long long* dst_ptr, const float* base, float* out, int N, int C, int Rk,
                                    float scale) {
  return maloq::edge_rotate_back_scatter(L, MM, Y, ldy, koff, rot, dst_ptr, base, out, N, C, Rk, scale, nullptr);
}

const char* emu_rotate_back_edge(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot, float* out,
                                 int E, int C, int Rk) {
  return maloq::edge_rotate_back(L, MM, Y, ldy, koff, rot, out, E, C, Rk, nullptr);
}

const char* emu_rotate_grad(int L, int MM, const float* G, const long long* rows, const float* rot, __nv_bfloat16* DY,
                            float* DYf, int E, int C, int Rk, float scale) {
  return maloq::edge_rotate_grad(L, MM, G, rows, rot, DY, DYf, E, C, Rk, scale, nullptr);
}

const char* emu_gate_fwd(int L, int MM, const __nv_bfloat16* Y1, __nv_bfloat16* H1, int E, int H) {
  return maloq::edge_gate_fwd(L, MM, Y1, H1, E, H, nullptr);
}

const char* emu_gate_bwd(int L, int MM, const __nv_bfloat16* Y1, const __nv_bfloat16* dH1, __nv_bfloat16* dY1, int E,
                         int H) {
  return maloq::edge_gate_bwd(L, MM, Y1, dH1, dY1, E, H, nullptr);
}

const char* emu_node_reduce(const float* DDST, const long long* dst_ptr, const float* DSRC, const long long* src_perm,
                            const long long* src_ptr, float* DX, int N, int SC, long long n_dst_rows,
                            long long n_src_rows) {
  return maloq::edge_node_reduce(DDST, dst_ptr, DSRC, src_perm, src_ptr, DX, N, SC, n_dst_rows, n_src_rows, nullptr);
}
}
