// A small CUDA-on-CPU runtime for tests: kernels from ops/csrc, rewritten textually by the test
// (launch syntax, shared-memory declarations, this header in place of common.cuh), run with one
// std::thread per CUDA thread of a block (one team per launch), blocks one after another.
//
// * __syncthreads: a barrier over the block's threads (threads that returned are dropped);
// * warp shuffles: a per-warp exchange buffer between two warp barriers;
// * dynamic shared memory: one zeroed buffer per block; static __shared__ arrays become
//   function statics (shared by the block's threads, blocks run one at a time);
// * __ldg: a plain load that first checks the address's alignment for the loaded type (a
//   misaligned float2 / float4 load faults on the GPU, so it aborts here);
// * the device error word: a host atomic.
#pragma once
#define MALOQ_EMU_RUNTIME 1
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <tuple>
#include <vector>

#ifndef MALOQ_SPIN_LIMIT
#define MALOQ_SPIN_LIMIT (1u << 26)
#endif

namespace emu {

struct Dim {
  unsigned x = 0, y = 0, z = 0;
};
inline thread_local Dim t_idx, b_idx;
inline Dim b_dim, g_dim;
inline thread_local int t_lin = 0;

struct Block {
  std::unique_ptr<std::barrier<>> bar;
  std::vector<std::unique_ptr<std::barrier<>>> warp;
  std::vector<float> shfl;
  std::vector<unsigned char> smem;
};
inline Block* block = nullptr;

inline void sync_block() { block->bar->arrive_and_wait(); }

template <class T>
inline T shfl_xor(T v, int lane_mask) {
  static_assert(sizeof(T) == sizeof(float), "emulated shuffles move 32-bit values");
  const int w = t_lin / 32, lane = t_lin % 32;
  float f;
  std::memcpy(&f, &v, sizeof f);
  block->shfl[w * 32 + lane] = f;
  block->warp[w]->arrive_and_wait();
  const float g = block->shfl[w * 32 + (lane ^ lane_mask)];
  block->warp[w]->arrive_and_wait();
  T out;
  std::memcpy(&out, &g, sizeof out);
  return out;
}

inline void* dyn_smem() { return block->smem.data(); }

inline std::atomic<int> error_word{0};

struct Cfg {
  dim3 grid, blk;
  size_t smem;
  Cfg(dim3 g, dim3 b, size_t s = 0, cudaStream_t = nullptr) : grid(g), blk(b), smem(s) {}
};

template <class... A>
struct Bound {
  void (*f)(A...);
  Cfg cfg;
};

template <class... A>
inline Bound<A...> operator^(void (*f)(A...), Cfg c) {
  return Bound<A...>{f, c};
}

template <class... T>
inline std::tuple<T...> args(T... t) {
  return std::tuple<T...>(t...);
}

// One team of nt host threads per launch walks the grid's blocks in order.  Between blocks the
// team meets at a barrier whose completion step (run by one thread while the others wait) re-arms
// the block's barriers - threads that returned from the kernel dropped out of them - clears the
// shared memory and moves to the next block index.
template <class... A, class... T>
inline void operator|(Bound<A...> b, std::tuple<T...> t) {
  const unsigned nt = b.cfg.blk.x * b.cfg.blk.y * b.cfg.blk.z;
  const unsigned long long nb = (unsigned long long)b.cfg.grid.x * b.cfg.grid.y * b.cfg.grid.z;
  if (nt == 0 || nb == 0) return;
  g_dim = Dim{b.cfg.grid.x, b.cfg.grid.y, b.cfg.grid.z};
  b_dim = Dim{b.cfg.blk.x, b.cfg.blk.y, b.cfg.blk.z};
  std::tuple<A...> a = std::apply([](auto... v) { return std::tuple<A...>(static_cast<A>(v)...); }, t);
  const unsigned nw = (nt + 31) / 32;
  Block blk;
  blk.shfl.assign(nw * 32, 0.f);
  auto arm = [&] {
    blk.bar = std::make_unique<std::barrier<>>(nt);
    blk.warp.clear();
    for (unsigned w = 0; w < nw; ++w) blk.warp.push_back(std::make_unique<std::barrier<>>(std::min(32u, nt - 32 * w)));
    blk.smem.assign(b.cfg.smem + 16, 0);
  };
  arm();
  block = &blk;
  unsigned long long cur = 0;
  auto next = [&]() noexcept {
    ++cur;
    if (cur < nb) arm();
  };
  std::barrier<decltype(next)> end(nt, next);
  std::vector<std::thread> th;
  th.reserve(nt);
  for (unsigned t = 0; t < nt; ++t)
    th.emplace_back([&, t] {
      t_lin = (int)t;
      t_idx = Dim{t % b.cfg.blk.x, (t / b.cfg.blk.x) % b.cfg.blk.y, t / (b.cfg.blk.x * b.cfg.blk.y)};
      for (unsigned long long q = 0; q < nb; ++q) {
        b_idx = Dim{(unsigned)(q % b.cfg.grid.x), (unsigned)((q / b.cfg.grid.x) % b.cfg.grid.y),
                    (unsigned)(q / ((unsigned long long)b.cfg.grid.x * b.cfg.grid.y))};
        std::apply(b.f, a);
        blk.warp[t / 32]->arrive_and_drop();
        blk.bar->arrive_and_drop();
        end.arrive_and_wait();
      }
    });
  for (auto& x : th) x.join();
  block = nullptr;
}

template <class T>
inline T ldg(const T* p) {
  if (reinterpret_cast<uintptr_t>(p) % alignof(T) != 0) {
    std::fprintf(stderr, "misaligned %zu-byte load at %p\n", sizeof(T), (const void*)p);
    std::abort();
  }
  return *p;
}

}  // namespace emu

#undef __launch_bounds__
#define __launch_bounds__(...)
#define threadIdx (::emu::t_idx)
#define blockIdx (::emu::b_idx)
#define blockDim (::emu::b_dim)
#define gridDim (::emu::g_dim)
#define __syncthreads() ::emu::sync_block()
#define __shfl_xor_sync(mask, v, o) ::emu::shfl_xor((v), (o))
#define __ldg(p) ::emu::ldg(p)
#undef cudaGetLastError
#define cudaGetLastError() cudaSuccess
#define cudaGetErrorString(e) "emulated launch error"
#undef __grid_constant__
#define __grid_constant__
// launch attributes have no effect on the emulated launch
#define cudaFuncSetAttribute(...) cudaSuccess

// device math names the kernels call, from their mathematical definitions
inline float rsqrtf(float x) { return 1.f / std::sqrt(x); }
inline float __expf(float x) { return std::exp(x); }
inline void sincosf_emu(float x, float* s, float* c) {
  *s = std::sin(x);
  *c = std::cos(x);
}
#define sincosf sincosf_emu

namespace maloq {

enum : int {
  ERR_NONE = 0,
  ERR_TMA_WAIT = 1,
  ERR_MMA_WAIT = 2,
  ERR_EPI_WAIT = 3,
  ERR_PEER_WAIT = 4,
  ERR_BOUNDS = 5,
};

inline void record_error(int code) {
  int z = 0;
  ::emu::error_word.compare_exchange_strong(z, code);
}

// the device code's fast exponential is CUDA's __expf; the host build uses the C library's expf
inline float silu(float x) { return x / (1.f + std::exp(-x)); }
inline float dsilu(float x) {
  const float s = 1.f / (1.f + std::exp(-x));
  return s * (1.f + x * (1.f - s));
}

#ifdef MALOQ_BOUNDS_CHECK
#define MALOQ_IN_BOUNDS(cond) ((cond) ? true : (::maloq::record_error(::maloq::ERR_BOUNDS), false))
#define MALOQ_BOUNDS_CHECKED 1
#else
#define MALOQ_IN_BOUNDS(cond) true
#define MALOQ_BOUNDS_CHECKED 0
#endif

}  // namespace maloq
