#pragma once
#include <cuda_runtime.h>

namespace maloq {

// One pass of the device radius graph over n_targets target atoms (global ids ``targets``).
// Atoms are binned into ncell[d] cells of width ext[d] / ncell[d] starting at lo[d]
// (``sorted_atoms`` grouped by flat cell id, ``cell_start`` [n_cells + 1]).  Count pass:
// counts[t] = sources within the cutoff; fill pass: src/vec at ptr[t] + k.
struct RadiusGraphArgs {
  const double* pos;  // [N, 3]
  const long long* targets;
  int n_targets;
  const long long* sorted_atoms;
  const long long* cell_start;
  double lo[3], ext[3];
  int ncell[3];
  int periodic[3];
  double cutoff;
  long long* counts;      // count pass
  const long long* ptr;   // fill pass: [n_targets] start offsets
  long long* src;         // fill pass
  double* vec;            // fill pass [E, 3]
};

const char* radius_graph_pass(const RadiusGraphArgs& a, bool fill, cudaStream_t st);
// flat cell id of each of the n_atoms atoms (same binning as the passes)
const char* radius_graph_cells(const RadiusGraphArgs& a, long long n_atoms, long long* cell, cudaStream_t st);

}  // namespace maloq
