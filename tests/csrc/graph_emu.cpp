// extern "C" entry points to the radius-graph launchers of graph.cu in the emulated build.
#include "graph_emu_src.inc"

extern "C" {
int emu_error_word() { return ::emu::error_word.exchange(0); }

// grid = (lo[3], ext[3], cutoff), ncell[3], periodic[3]
static maloq::RadiusGraphArgs args_of(const double* pos, const double* grid, const int* ncell, const int* periodic) {
  maloq::RadiusGraphArgs a{};
  a.pos = pos;
  for (int d = 0; d < 3; ++d) {
    a.lo[d] = grid[d];
    a.ext[d] = grid[3 + d];
    a.ncell[d] = ncell[d];
    a.periodic[d] = periodic[d];
  }
  a.cutoff = grid[6];
  return a;
}

const char* emu_radius_graph_cells(const double* pos, long long n, const double* grid, const int* ncell,
                                   const int* periodic, long long* cell) {
  return maloq::radius_graph_cells(args_of(pos, grid, ncell, periodic), n, cell, nullptr);
}

const char* emu_radius_graph_pass(const double* pos, const double* grid, const int* ncell, const int* periodic,
                                  const long long* targets, int n_targets, const long long* sorted_atoms,
                                  const long long* cell_start, long long* counts, const long long* ptr,
                                  long long* src, double* vec, int fill) {
  maloq::RadiusGraphArgs a = args_of(pos, grid, ncell, periodic);
  a.targets = targets;
  a.n_targets = n_targets;
  a.sorted_atoms = sorted_atoms;
  a.cell_start = cell_start;
  a.counts = counts;
  a.ptr = ptr;
  a.src = src;
  a.vec = vec;
  return maloq::radius_graph_pass(a, fill != 0, nullptr);
}
}
