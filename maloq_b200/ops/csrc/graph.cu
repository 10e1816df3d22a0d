// Radius graph on the device: cell list, periodic (orthorhombic, minimum image) or open.
//
// The host side bins atoms into cells of edge >= cutoff and sorts them by cell (torch ops);
// here one thread per target atom walks the (deduplicated) 27 neighbour cells twice: a count
// pass sizes each target's edge range, a fill pass writes (source, pos[src] - pos[dst]) into it.
// Distances are evaluated in fp64 so the cutoff test agrees with the host builder.  Reference
// behaviour: ASE NeighborList on the host (fock_utils/fock_targets_batched.py:189-229).
#include "common.cuh"
#include "graph.h"

namespace maloq {

struct CellGrid {
  double lo[3], ext[3], width[3];  // grid origin, extent (the cell for periodic axes), cell width
  int n[3];                        // cells per axis
  int periodic[3];
  double cut2;
};

__device__ __forceinline__ int cell_coord(double p, double lo, double w, int n) {
  int c = (int)floor((p - lo) / w);
  return c < 0 ? 0 : (c >= n ? n - 1 : c);
}

// Unique neighbour-cell offsets along one axis: {-1,0,1}, or fewer when wrapping (periodic,
// n < 3) or clipping (open boundary) would visit a cell twice or leave the grid.
__device__ __forceinline__ int axis_offsets(int c, int n, int periodic, int* out) {
  int k = 0;
  for (int o = -1; o <= 1; ++o) {
    int v = c + o;
    if (periodic) {
      v = ((v % n) + n) % n;
      bool dup = false;
      for (int q = 0; q < k; ++q) dup |= out[q] == v;
      if (!dup) out[k++] = v;
    } else if (v >= 0 && v < n) {
      out[k++] = v;
    }
  }
  return k;
}

__device__ __forceinline__ int wrapped_cell(double p, const CellGrid& G, int d) {
  const double q = G.periodic[d] ? p - G.ext[d] * floor((p - G.lo[d]) / G.ext[d]) : p;
  return cell_coord(q, G.lo[d], G.width[d], G.n[d]);
}

// flat cell id of every atom (the host sorts atoms by it)
__global__ void cell_id_kernel(const double* __restrict__ pos, long long n, const __grid_constant__ CellGrid G,
                               long long* __restrict__ cell) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int cx = wrapped_cell(pos[3 * i], G, 0), cy = wrapped_cell(pos[3 * i + 1], G, 1),
            cz = wrapped_cell(pos[3 * i + 2], G, 2);
  cell[i] = ((long long)cx * G.n[1] + cy) * G.n[2] + cz;
}

template <bool FILL>
__global__ void radius_graph_kernel(const double* __restrict__ pos, const long long* __restrict__ targets, int n_t,
                                    const long long* __restrict__ sorted_atoms, const long long* __restrict__ cell_start,
                                    const __grid_constant__ CellGrid G, long long* __restrict__ counts,
                                    const long long* __restrict__ ptr, long long* __restrict__ src_out,
                                    double* __restrict__ vec_out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_t) return;
  const long long i = targets[t];
  const double px = pos[3 * i], py = pos[3 * i + 1], pz = pos[3 * i + 2];
  int ox[3], oy[3], oz[3];
  const int nx = axis_offsets(wrapped_cell(px, G, 0), G.n[0], G.periodic[0], ox);
  const int ny = axis_offsets(wrapped_cell(py, G, 1), G.n[1], G.periodic[1], oy);
  const int nz = axis_offsets(wrapped_cell(pz, G, 2), G.n[2], G.periodic[2], oz);
  long long k = FILL ? ptr[t] : 0;
  for (int a = 0; a < nx; ++a)
    for (int b = 0; b < ny; ++b)
      for (int c = 0; c < nz; ++c) {
        const long long cell = ((long long)ox[a] * G.n[1] + oy[b]) * G.n[2] + oz[c];
        for (long long s = cell_start[cell]; s < cell_start[cell + 1]; ++s) {
          const long long j = sorted_atoms[s];
          if (j == i) continue;
          double dx = pos[3 * j] - px, dy = pos[3 * j + 1] - py, dz = pos[3 * j + 2] - pz;
          if (G.periodic[0]) dx -= G.ext[0] * rint(dx / G.ext[0]);
          if (G.periodic[1]) dy -= G.ext[1] * rint(dy / G.ext[1]);
          if (G.periodic[2]) dz -= G.ext[2] * rint(dz / G.ext[2]);
          if (dx * dx + dy * dy + dz * dz >= G.cut2) continue;
          if (FILL) {
            src_out[k] = j;
            vec_out[3 * k] = dx;
            vec_out[3 * k + 1] = dy;
            vec_out[3 * k + 2] = dz;
          }
          ++k;
        }
      }
  if (!FILL) counts[t] = k;
}

static CellGrid make_grid(const RadiusGraphArgs& a) {
  CellGrid G;
  for (int d = 0; d < 3; ++d) {
    G.lo[d] = a.lo[d];
    G.ext[d] = a.ext[d];
    G.n[d] = a.ncell[d];
    G.width[d] = a.ext[d] / a.ncell[d];
    G.periodic[d] = a.periodic[d];
  }
  G.cut2 = a.cutoff * a.cutoff;
  return G;
}

const char* radius_graph_cells(const RadiusGraphArgs& a, long long n_atoms, long long* cell, cudaStream_t st) {
  if (n_atoms == 0) return nullptr;
  const CellGrid G = make_grid(a);
  cell_id_kernel<<<(unsigned)((n_atoms + 255) / 256), 256, 0, st>>>(a.pos, n_atoms, G, cell);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

const char* radius_graph_pass(const RadiusGraphArgs& a, bool fill, cudaStream_t st) {
  if (a.n_targets == 0) return nullptr;
  const CellGrid G = make_grid(a);
  const int threads = 128;
  const unsigned blocks = (unsigned)((a.n_targets + threads - 1) / threads);
  if (fill)
    radius_graph_kernel<true><<<blocks, threads, 0, st>>>(a.pos, a.targets, a.n_targets, a.sorted_atoms,
                                                          a.cell_start, G, nullptr, a.ptr, a.src, a.vec);
  else
    radius_graph_kernel<false><<<blocks, threads, 0, st>>>(a.pos, a.targets, a.n_targets, a.sorted_atoms,
                                                           a.cell_start, G, a.counts, nullptr, nullptr, nullptr);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace maloq
