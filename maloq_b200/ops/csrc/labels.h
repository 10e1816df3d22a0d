#pragma once
#include <cuda_runtime.h>

namespace maloq {

// Row transform out[r, u] = sum_{j < n_u} in[r, s_u + j] * coef[c_u + j * n_u] for the columns
// u of a block-diagonal (coupled <-> uncoupled) basis transform, described per output column by
// meta[u] = (s_u, n_u, c_u, 0).
//   gather:  in[r, k] = data[ptr[r] + pos[pt[r] * d_pos + k]]  (0 where pos < 0)
//   scatter: data[ptr[r] + pos[pt[r] * d_pos + u]] = out[r, u] (skipped where pos < 0)
// Otherwise rows are dense with leading dimension ld_in / ld_out.  dtype 0 = fp32, 1 = fp64.
struct BasisRowsArgs {
  const void* in;
  long long ld_in;
  void* out;
  long long ld_out;
  const long long* ptr;  // [rows] block offsets (gather or scatter)
  const long long* pt;   // [rows] pair types
  const int* pos;        // [n_pair_types, d_pos]
  int d_pos;
  const int4* meta;      // [d_out]
  const void* coef;
  int d_in, d_out;
  long long rows;
  long long n_pt;    // rows of the position table (bounds checks)
  long long n_data;  // entries of the block data (bounds checks)
  bool gather, scatter;
  int dtype;
};

const char* basis_rows(const BasisRowsArgs& a, cudaStream_t st);

}  // namespace maloq
