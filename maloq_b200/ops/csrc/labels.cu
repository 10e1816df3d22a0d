// Hamiltonian block <-> label row conversion fused with the coupled <-> uncoupled basis
// transform.
//
// The transform matrix is block diagonal: every orbital shell pair (l1, l2) owns a square
// (2l1+1)(2l2+1) block (Clebsch-Gordan / Wigner-3j coefficients; reference
// fock_utils/utils_tensor_decomp.py:51-169 multiplies by the dense [D, D] matrix, and the Triton
// backend basis_transform_triton_backend.py:33-154 by the blocks).  Block-sparse Hamiltonian data
// <-> label rows goes through a per element-pair position table (reference
// fock_utils/matrix2labels_kernels.py:689-800 copies with one CTA per block).
//
// Here one kernel does gather -> transform -> scatter for a tile of ROWS label rows:
//   1. the tile's input rows are staged in shared memory (gathered from the block data through
//      the position table, or read as dense rows);
//   2. each thread owns output columns; column u is a dot product of length n_u <= 49 over the
//      staged inputs of its CG block, each coefficient loaded once and used for all ROWS rows
//      (coefficients of adjacent columns are adjacent, so a warp's loads coalesce);
//   3. results go to dense rows or are scattered into the block data.
// The work is memory bound (a few FLOP per byte), so it runs on the fp32/fp64 pipes at the
// reference's precision rather than on tensor cores.  The identity transform (n_u = 1) gives
// the plain matrix <-> label copies.
#include "common.cuh"
#include "labels.h"

namespace maloq {

constexpr int BT_ROWS = 8;
constexpr int BT_THREADS = 256;

template <typename T, bool GATHER, bool SCATTER>
__global__ void __launch_bounds__(BT_THREADS) basis_rows_kernel(const T* __restrict__ in, long long ld_in,
                                                                T* __restrict__ out, long long ld_out,
                                                                const long long* __restrict__ ptr,
                                                                const long long* __restrict__ pt,
                                                                const int* __restrict__ pos, int d_pos,
                                                                const int4* __restrict__ meta,
                                                                const T* __restrict__ coef, int d_in, int d_out,
                                                                long long rows, long long n_pt, long long n_data) {
  extern __shared__ __align__(16) unsigned char bt_smem[];
  T* xs = reinterpret_cast<T*>(bt_smem);  // [BT_ROWS][d_in]
  const long long n_tiles = (rows + BT_ROWS - 1) / BT_ROWS;
  for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const long long r0 = tile * BT_ROWS;
    for (int idx = threadIdx.x; idx < BT_ROWS * d_in; idx += BT_THREADS) {
      const int r = idx / d_in, k = idx - r * d_in;
      const long long row = r0 + r;
      T v = T(0);
      if (row < rows) {
        if (GATHER) {
          // a failed check skips the access only: every thread still reaches the barriers below
          const long long t = __ldg(pt + row);
          if (MALOQ_IN_BOUNDS(t >= 0 && t < n_pt)) {
            const int p = __ldg(pos + t * d_pos + k);
            if (p >= 0 && MALOQ_IN_BOUNDS(__ldg(ptr + row) + p < n_data)) v = in[__ldg(ptr + row) + p];
          }
        } else {
          v = in[row * ld_in + k];
        }
      }
      xs[r * d_in + k] = v;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < d_out; u += BT_THREADS) {
      const int4 m = __ldg(meta + u);
      T acc[BT_ROWS];
#pragma unroll
      for (int r = 0; r < BT_ROWS; ++r) acc[r] = T(0);
      for (int j = 0; j < m.y; ++j) {
        const T c = __ldg(coef + m.z + j * m.y);
#pragma unroll
        for (int r = 0; r < BT_ROWS; ++r) acc[r] += xs[r * d_in + m.x + j] * c;
      }
#pragma unroll
      for (int r = 0; r < BT_ROWS; ++r) {
        const long long row = r0 + r;
        if (row >= rows) break;
        if (SCATTER) {
          const long long t = __ldg(pt + row);
          if (MALOQ_IN_BOUNDS(t >= 0 && t < n_pt)) {
            const int p = __ldg(pos + t * d_pos + u);
            if (p >= 0 && MALOQ_IN_BOUNDS(__ldg(ptr + row) + p < n_data)) out[__ldg(ptr + row) + p] = acc[r];
          }
        } else {
          out[row * ld_out + u] = acc[r];
        }
      }
    }
    __syncthreads();
  }
}

template <typename T, bool G, bool S>
static void launch_bt(const BasisRowsArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(T) * BT_ROWS * (size_t)a.d_in;
  auto k = basis_rows_kernel<T, G, S>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const long long tiles = (a.rows + BT_ROWS - 1) / BT_ROWS;
  const int grid = (int)std::min<long long>(tiles, 148LL * 8);
  k<<<grid, BT_THREADS, smem, st>>>(static_cast<const T*>(a.in), a.ld_in, static_cast<T*>(a.out), a.ld_out, a.ptr,
                                    a.pt, a.pos, a.d_pos, a.meta, static_cast<const T*>(a.coef), a.d_in, a.d_out,
                                    a.rows, a.n_pt, a.n_data);
}

template <typename T>
static void dispatch_bt(const BasisRowsArgs& a, cudaStream_t st) {
  if (a.gather && a.scatter) launch_bt<T, true, true>(a, st);
  else if (a.gather) launch_bt<T, true, false>(a, st);
  else if (a.scatter) launch_bt<T, false, true>(a, st);
  else launch_bt<T, false, false>(a, st);
}

const char* basis_rows(const BasisRowsArgs& a, cudaStream_t st) {
  const size_t esz = a.dtype == 1 ? 8 : 4;
  if (esz * BT_ROWS * (size_t)a.d_in > 200 * 1024) return "basis_rows: input row too wide for shared memory";
  if ((a.gather || a.scatter) && (a.ptr == nullptr || a.pt == nullptr || a.pos == nullptr))
    return "basis_rows: gather/scatter needs ptr, pair types and the position table";
  if (a.rows == 0 || a.d_out == 0) return nullptr;
  if (a.dtype == 1) dispatch_bt<double>(a, st);
  else dispatch_bt<float>(a, st);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace maloq
