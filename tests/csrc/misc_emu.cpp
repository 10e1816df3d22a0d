// extern "C" entry points to the host launchers of misc.cu (edge rotation, Fock loss, radial
// inputs, column sums, weight packing) in the emulated build; the test compiles this file after rewriting misc.cu for
// tests/csrc/host_emu.cuh.
#include "misc_emu_src.inc"

extern "C" {
int emu_error_word() { return ::emu::error_word.exchange(0); }

const char* emu_edge_rotation(const float* vec, long long ldv, const float* J, const int* joff, int L,
                              const int* row_l, const int* row_m, int R, float* ROT, int E) {
  return maloq::edge_rotation(vec, ldv, J, joff, L, row_l, row_m, R, ROT, E, nullptr);
}

int emu_fock_loss_grid(long long n) { return maloq::fock_loss_grid(n); }

const char* emu_fock_loss_stats(const float* O, const float* T, const long long* pt, const uint8_t* mask, int D,
                                long long rows, float* part, int grid, long long n_pt) {
  return maloq::fock_loss_stats(O, T, pt, mask, D, rows, part, grid, n_pt, nullptr);
}

const char* emu_fock_loss_grad(const float* O, const float* T, const long long* pt, const uint8_t* mask, int D,
                               long long rows, const float* gstat, float* G, long long n_pt) {
  return maloq::fock_loss_grad(O, T, pt, mask, D, rows, gstat, G, n_pt, nullptr);
}

const char* emu_edge_inputs(const long long* src_z, const long long* dst_z, const float* D, long long ld_d,
                            const float* src_table, const float* dst_table, long long n_types, const float* offset,
                            float coeff, __nv_bfloat16* OUT, long long E, int C, int NB) {
  return maloq::edge_inputs(src_z, dst_z, D, ld_d, src_table, dst_table, n_types, offset, coeff, OUT, E, C, NB,
                            nullptr);
}

int emu_colsum_chunks(long long M, int N) { return maloq::colsum_chunks(M, N); }

const char* emu_colsum(const void* X, int bf16, long long M, int N, long long ld, float* part, int P, float* out) {
  return maloq::colsum(X, bf16 != 0, M, N, ld, part, P, out, nullptr);
}

const char* emu_weight_pack(int n, const float* const* src, void* const* dst, const int* batch, const int* rows,
                            const int* cols, const int* kind) {
  return maloq::weight_pack(n, src, dst, batch, rows, cols, kind, nullptr);
}

const char* emu_colsum_segments(const float* X, int N, long long ld, const long long* seg, int nseg, float* out) {
  return maloq::colsum_segments(X, N, ld, seg, nseg, out, nullptr);
}
}
