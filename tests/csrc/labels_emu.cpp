// extern "C" entry point to the basis-row launcher of labels.cu in the emulated build.
#include "labels_emu_src.inc"

extern "C" {
int emu_error_word() { return ::emu::error_word.exchange(0); }

const char* emu_basis_rows(const void* in, long long ld_in, void* out, long long ld_out, const long long* ptr,
                           const long long* pt, const int* pos, int d_pos, const int* meta, const void* coef, int d_in,
                           int d_out, long long rows, long long n_pt, long long n_data, int gather, int scatter,
                           int dtype) {
  maloq::BasisRowsArgs a;
  a.in = in;
  a.ld_in = ld_in;
  a.out = out;
  a.ld_out = ld_out;
  a.ptr = ptr;
  a.pt = pt;
  a.pos = pos;
  a.d_pos = d_pos;
  a.meta = reinterpret_cast<const int4*>(meta);
  a.coef = coef;
  a.d_in = d_in;
  a.d_out = d_out;
  a.rows = rows;
  a.n_pt = n_pt;
  a.n_data = n_data;
  a.gather = gather != 0;
  a.scatter = scatter != 0;
  a.dtype = dtype;
  return maloq::basis_rows(a, nullptr);
}
}
