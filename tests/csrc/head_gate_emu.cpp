// Host build of the Fock-head gate kernels (maloq_b200/ops/csrc/head_gate.cuh): each kernel runs
// over an emulated grid, one (block, thread) pair at a time, on the CPU.  Used by
// tests/test_kernel_emulation.py to check the kernels' index arithmetic and math against PyTorch
// on a machine without a GPU.
#define MALOQ_HOST_EMULATION 1
struct EmuDim {
  unsigned x = 0, y = 0, z = 0;
};
static EmuDim blockIdx, threadIdx, blockDim, gridDim;

#include "head_gate.cuh"

template <class F>
static void run_grid(int grid, int block, F&& body) {
  gridDim.x = grid;
  blockDim.x = block;
  for (int b = 0; b < grid; ++b)
    for (int t = 0; t < block; ++t) {
      blockIdx.x = b;
      threadIdx.x = t;
      body();
    }
}

#define EMU_L(L_, ...) \
  case L_: {           \
    constexpr int LL = L_; \
    __VA_ARGS__;       \
    return 0;          \
  }
#define EMU_DISPATCH(...)                                                                                 \
  switch (L) {                                                                                            \
    EMU_L(0, __VA_ARGS__) EMU_L(1, __VA_ARGS__) EMU_L(2, __VA_ARGS__) EMU_L(3, __VA_ARGS__)             \
    EMU_L(4, __VA_ARGS__) EMU_L(5, __VA_ARGS__) EMU_L(6, __VA_ARGS__) default: return 1;              \
  }

extern "C" int emu_head_gate_fwd(int L, const float* X, const float* SV, __nv_bfloat16* A, int act, float scale,
                                 int absg, int B, int C, int grid, int block) {
  if (act == 0) {
    EMU_DISPATCH(run_grid(grid, block, [&] { maloq::head_gate_fwd_kernel<LL, 0>(X, SV, A, B, C, scale, absg); }))
  }
  EMU_DISPATCH(run_grid(grid, block, [&] { maloq::head_gate_fwd_kernel<LL, 1>(X, SV, A, B, C, scale, absg); }))
}

extern "C" int emu_head_gate_bwd(int L, const float* X, const float* SV, const float* DA, float* DX, float* DSV,
                                 int act, float scale, int absg, int B, int C, int grid, int block) {
  if (act == 0) {
    EMU_DISPATCH(run_grid(grid, block, [&] { maloq::head_gate_bwd_kernel<LL, 0>(X, SV, DA, DX, DSV, B, C, scale, absg); }))
  }
  EMU_DISPATCH(run_grid(grid, block, [&] { maloq::head_gate_bwd_kernel<LL, 1>(X, SV, DA, DX, DSV, B, C, scale, absg); }))
}
