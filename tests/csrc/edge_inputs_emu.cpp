// Host build of the radial-input kernel (maloq_b200/ops/csrc/edge_inputs.cuh) over an emulated
// grid, for tests/test_kernel_emulation.py.
#define MALOQ_HOST_EMULATION 1
struct EmuDim {
  unsigned x = 0, y = 0, z = 0;
};
static EmuDim blockIdx, threadIdx, blockDim, gridDim;

#include "edge_inputs.cuh"

extern "C" int emu_edge_inputs(const long long* src_z, const long long* dst_z, const float* D, long long ld_d,
                               const float* src_table, const float* dst_table, long long n_types, const float* offset,
                               float coeff, __nv_bfloat16* out, long long E, int C, int NB, int grid, int block) {
  maloq::g_emulated_error = 0;
  gridDim.x = grid;
  blockDim.x = block;
  for (int b = 0; b < grid; ++b)
    for (int t = 0; t < block; ++t) {
      blockIdx.x = b;
      threadIdx.x = t;
      maloq::edge_inputs_kernel(src_z, dst_z, D, ld_d, src_table, dst_table, n_types, offset, coeff, out, E, C, NB);
    }
  return maloq::g_emulated_error;
}
