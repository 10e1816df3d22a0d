// Grouped bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   C[p] (M x N) = alpha * A[p] (M x K) * B[p]^T (K x N) (+ bias[N]) (act) (+ R[p])
//
// R (optional, fp32 output only, no split-K) is a residual read in the epilogue: a row-major
// [M, N] view with its own row stride, added after the activation.
//
// A and B are bf16 and either K-major (row-major [M,K] / [N,K]) or MN-major (row-major
// [K,M] / [K,N], used for weight gradients where K is the edge dimension).  Up to eight
// problems run in one launch (the per-|m| SO(2) GEMMs of a layer).  Optional split-K
// writes fp32 partials [split][M][N]; gemm_splitk_reduce sums them in a fixed order, so
// weight gradients are deterministic.
//
// Persistent CTAs (one per SM) walk a static schedule of 128 x BN output tiles; K in steps of
// 64 through a STAGES-deep TMA ring:
//   warp 0 (one elected lane): TMA producer        - waits "empty", loads the A/B tiles
//   warp 1 (one elected lane): tcgen05.mma issuer  - waits "full", 4 MMAs (K=16), commits "empty"
//   warps 2-9: epilogue - tcgen05.ld of TMEM lanes 32*(w%4).. (two warps per lane quarter, each
//   half of the columns), bias/activation/residual, store.
// Two TMEM accumulators (2 x BN fp32 columns) let a tile's epilogue overlap the next tile's
// MMAs.  TMA loads use no multicast.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm.h"

namespace maloq {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int EPI_WARPS = 8;             // two warps per TMEM lane quarter, each half of the columns
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int STAGE_WARP_BYTES = 8192;   // epilogue staging per epilogue warp

struct alignas(64) GemmProblemDev {
  CUtensorMap ta;
  CUtensorMap tb;
  CUtensorMap tc;  // output, 3-D {N, M, splits}, box {32, 32, 1}, swizzled
  void* c;
  const float* bias;
  const float* resid;
  long long ldc;
  long long ldr;
  long long split_stride;
  int M, N, K;
  int tiles_n;
  int tile_begin;
  int k_per_split;
};

struct GemmParamsDev {
  GemmProblemDev p[8];
  int nprob;
  int out_fp32;
  int act;
  float alpha;
};

// Decode a linear work index into (problem, m0, n0, split).
struct TileCoord {
  int pi, m0, n0, split;
};

// Epilogue scalars of one work item, copied out of the parameter block into registers once
// per tile (reading them through a reference into the grid-constant block inside the chunk
// loop costs a parameter-window load per use).
struct EpiScalars {
  const float* bias;
  float alpha;
  int act, N, M;
  const float* resid;
  long long ldr;
};

// v[j] += R[row, col0 + j] (the residual of the lane's row; 32 consecutive floats)
__device__ __forceinline__ void epilogue_residual(float* v, const EpiScalars& ep, int row, int col0) {
  if (ep.resid == nullptr || row >= ep.M) return;
  const float* r = ep.resid + (size_t)row * ep.ldr + col0;
  if (col0 + 32 <= ep.N && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(r) + j);
      v[4 * j] += t.x;
      v[4 * j + 1] += t.y;
      v[4 * j + 2] += t.z;
      v[4 * j + 3] += t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < ep.N) v[j] += __ldg(r + j);
  }
}

// v[j] (column col0 + j of this lane's row) = act(alpha * v[j] + bias[col0 + j]); lane j loads
// bias[col0 + j] and the row's 32 values are broadcast by shuffles.
__device__ __forceinline__ void epilogue_math(float* v, float alpha, const EpiScalars& ep, int col0, int lane) {
  float b = 0.f;
  if (ep.bias != nullptr && col0 + lane < ep.N) b = __ldg(ep.bias + col0 + lane);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = v[j] * alpha + __shfl_sync(0xffffffffu, b, j);
  if (ep.act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]);
  }
}

__device__ __forceinline__ TileCoord decode_tile(const GemmParamsDev& P, int w, int tiles_per_split, int BN,
                                                 int bm = BM) {
  TileCoord tc;
  tc.split = w / tiles_per_split;
  int t = w - tc.split * tiles_per_split;
  int pi = 0;
#pragma unroll 1
  for (int q = 1; q < P.nprob; ++q)
    if (t >= P.p[q].tile_begin) pi = q;
  t -= P.p[pi].tile_begin;
  tc.pi = pi;
  tc.m0 = (t / P.p[pi].tiles_n) * bm;
  tc.n0 = (t % P.p[pi].tiles_n) * BN;
  return tc;
}

// Persistent warp-specialised kernel: 10 warps.
//   warp 0: TMA producer (one lane); warp 1: MMA issuer (one lane);
//   warps 2-9: epilogue (warp w reads TMEM lanes 32*(w%4) .. +31, columns of its half).
// Two TMEM accumulators (2*BN columns): the epilogue of work item i overlaps the MMAs of i+1.
template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_tc_kernel(const __grid_constant__ GemmParamsDev P, int total_work,
                                                         int tiles_per_split) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;   // [2] epilogue -> MMA (one arrival per epilogue warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  // epilogue staging: EPI_WARPS x STAGE_WARP_BYTES, 1024-aligned
  uint8_t* stage_out = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tmem_slot + 4) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < P.nprob; ++q) {
      prefetch_tmap(&P.p[q].ta);
      prefetch_tmap(&P.p[q].tb);
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer
    if (elect_one()) {
      int kc = 0;  // k-tile counter across work items (stage ring position)
      for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x) {
        const TileCoord tc = decode_tile(P, w, tiles_per_split, BN);
        const GemmProblemDev& pr = P.p[tc.pi];
        const int k_begin = tc.split * pr.k_per_split;
        const int k_end = min(pr.K, k_begin + pr.k_per_split);
        const int k_tiles = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          if (kc >= STAGES && !mbar_wait(&empty[s], ((kc / STAGES) - 1) & 1, ERR_TMA_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
          const int k = k_begin + kt * BK;
          uint8_t* a = sA + s * A_BYTES;
          uint8_t* b = sB + s * B_BYTES;
          if constexpr (A_MN) {
            tma_load_2d(a, &pr.ta, &full[s], tc.m0, k);
            tma_load_2d(a + BK * 128, &pr.ta, &full[s], tc.m0 + 64, k);
          } else {
            tma_load_2d(a, &pr.ta, &full[s], k, tc.m0);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * BK * 128, &pr.tb, &full[s], tc.n0 + 64 * j, k);
          } else {
            tma_load_2d(b, &pr.tb, &full[s], k, tc.n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int kc = 0, it = 0;
      for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x, ++it) {
        const TileCoord tc = decode_tile(P, w, tiles_per_split, BN);
        const GemmProblemDev& pr = P.p[tc.pi];
        const int k_begin = tc.split * pr.k_per_split;
        const int k_end = min(pr.K, k_begin + pr.k_per_split);
        const int k_tiles = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
        const int buf = it & 1;
        if (it >= 2 && !mbar_wait(&acc_empty[buf], ((it >> 1) - 1) & 1, ERR_MMA_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          if (!mbar_wait(&full[s], (kc / STAGES) & 1, ERR_MMA_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * A_BYTES);
          const uint32_t b = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t ad, bd;
            if constexpr (A_MN) ad = sw128_desc(a + kk * 16 * 128, BK * 128, 1024);
            else ad = sw128_desc(a + kk * 32, 16, 1024);
            if constexpr (B_MN) bd = sw128_desc(b + kk * 16 * 128, BK * 128, 1024);
            else bd = sw128_desc(b + kk * 32, 16, 1024);
            umma_f16(d, ad, bd, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);  // also fires for k_tiles == 0 (epilogue writes zeros)
      }
    }
  } else {
    // ---------------- epilogue warps 2..9: warp w reads TMEM lanes 32*(w%4).. and half (w-2)/4 of
    // the accumulator's columns
    const int ew = warp - 2, quarter = warp & 3;
    const int cbeg = (ew / 4) * (BN / 2), cend = cbeg + BN / 2;
    const bool out32 = P.out_fp32 != 0;
    int it = 0, sbuf = 0;
    for (int w = blockIdx.x; w < total_work; w += gridDim.x, ++it) {
      const TileCoord tc = decode_tile(P, w, tiles_per_split, BN);
      const GemmProblemDev& pr = P.p[tc.pi];
      const EpiScalars ep{pr.bias, P.alpha, P.act, pr.N, pr.M, pr.resid, pr.ldr};
      const int k_begin = tc.split * pr.k_per_split;
      const bool have_k = min(pr.K, k_begin + pr.k_per_split) > k_begin;
      const int buf = it & 1;
      if (!mbar_wait(&acc_full[buf], (it >> 1) & 1, ERR_EPI_WAIT)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        if (c0 + 32 >= cend) {
          // this warp's part of the accumulator is read: hand it back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        const int col0 = tc.n0 + c0;
        if (col0 >= ep.N) continue;  // warp-uniform
        if (!have_k) {
          // a split with no k-tiles: no MMA wrote this accumulator, so its TMEM holds stale bits
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        epilogue_math(v, ep.alpha, ep, col0, lane);
        epilogue_residual(v, ep, tc.m0 + quarter * 32 + lane, col0);
        // stage the warp's 32 x 32 chunk (row-major, 32*esz bytes per row) and TMA-store it
        // per-warp ring of staging chunks (8 KB): 4 bf16 or 2 fp32 chunks of 32 x 32
        const int ring = out32 ? 2 : 4;
        uint8_t* stg = stage_out + ew * STAGE_WARP_BYTES + (sbuf % ring) * (out32 ? 4096 : 2048);
        if (lane == 0) {
          if (out32) bulk_wait_read<1>();  // the chunk stored `ring` chunks ago has been read
          else bulk_wait_read<3>();
        }
        __syncwarp();
        if (out32) {
          // 128B-swizzled staging: 16B chunk j of row r lives at chunk j ^ (r & 7)
          float4* dst = reinterpret_cast<float4*>(stg + lane * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          // 64B-swizzled staging: 16B chunk j of row r lives at chunk j ^ ((r >> 1) & 3)
          uint4* dst = reinterpret_cast<uint4*>(stg + lane * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
            dst[j ^ ((lane >> 1) & 3)] = *reinterpret_cast<uint4*>(h);
          }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0 && tc.m0 + quarter * 32 < ep.M) {
          tma_store_3d(&pr.tc, stg, col0, tc.m0 + quarter * 32, tc.split);
          bulk_commit();
        }
        ++sbuf;
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// ======================================================================= 2-SM variant
// A CTA pair (cluster of 2) computes a 256 x BN tile with tcgen05.mma.cta_group::2: CTA r
// loads rows [m0 + 128 r, +128) of A and rows [n0 + r BN/2, +BN/2) of B into its own shared
// memory; the leader (r = 0) issues the M = 256 MMAs, which read both CTAs' shared memory and
// write rows 128 r.. of the accumulator into CTA r's TMEM.  Per SM this halves the B bytes per
// FLOP relative to the 1-SM kernel.  K-major operands only; no split-K.
// Barriers: full[s] lives in the leader (both CTAs' TMA loads complete on it); empty[s] and
// acc_full[b] exist in both CTAs and are signalled by two commits from the leader; acc_empty[b]
// lives in the leader and collects 2 * EPI_WARPS arrivals (the epilogue warps of both CTAs).
template <int BN, int STAGES>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_tc2_kernel(const __grid_constant__ GemmParamsDev P, int total_work) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = 128 * BK * 2;
  constexpr int B_BYTES = (BN / 2) * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint8_t* stage_out = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tmem_slot + 4) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t crank = cluster_ctarank();
  const int cluster = blockIdx.x / 2, nclusters = gridDim.x / 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < P.nprob; ++q) {
      prefetch_tmap(&P.p[q].ta);
      prefetch_tmap(&P.p[q].tb);
    }
  }
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (elect_one()) {
      int kc = 0;
      for (int w = cluster; w < total_work && ok; w += nclusters) {
        const TileCoord tc = decode_tile(P, w, total_work, BN, 256);
        const GemmProblemDev& pr = P.p[tc.pi];
        const int k_tiles = (pr.K + BK - 1) / BK;
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          if (kc >= STAGES && !mbar_wait(&empty[s], ((kc / STAGES) - 1) & 1, ERR_TMA_WAIT)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = mapa_shared(smem_u32(&full[s]), 0);
          if (crank == 0) mbar_arrive_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
          const int k = kt * BK;
          tma_load_2d_pair(sA + s * A_BYTES, &pr.ta, leader_full, k, tc.m0 + 128 * (int)crank);
          tma_load_2d_pair(sB + s * B_BYTES, &pr.tb, leader_full, k, tc.n0 + (BN / 2) * (int)crank);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only)
    if (crank == 0 && elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(256, BN, 0, 0);
      const uint32_t empty0 = mapa_shared(smem_u32(&empty[0]), 0), empty1 = mapa_shared(smem_u32(&empty[0]), 1);
      const uint32_t accf0 = mapa_shared(smem_u32(&acc_full[0]), 0), accf1 = mapa_shared(smem_u32(&acc_full[0]), 1);
      int kc = 0, it = 0;
      for (int w = cluster; w < total_work && ok; w += nclusters, ++it) {
        const TileCoord tc = decode_tile(P, w, total_work, BN, 256);
        const GemmProblemDev& pr = P.p[tc.pi];
        const int k_tiles = (pr.K + BK - 1) / BK;
        const int buf = it & 1;
        if (it >= 2 && !mbar_wait(&acc_empty[buf], ((it >> 1) - 1) & 1, ERR_MMA_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          if (!mbar_wait(&full[s], (kc / STAGES) & 1, ERR_MMA_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * A_BYTES);
          const uint32_t b = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_pair(d, sw128_desc(a + kk * 32, 16, 1024), sw128_desc(b + kk * 32, 16, 1024), idesc,
                          (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(empty0 + s * 8);
          umma_commit_pair(empty1 + s * 8);
        }
        if (!ok) break;
        umma_commit_pair(accf0 + buf * 8);
        umma_commit_pair(accf1 + buf * 8);
      }
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs; rows 128 * crank + ...); warp w reads TMEM
    // lanes 32*(w%4).. and half (w-2)/4 of the columns
    const int ew = warp - 2, quarter = warp & 3;
    const int cbeg = (ew / 4) * (BN / 2), cend = cbeg + BN / 2;
    const bool out32 = P.out_fp32 != 0;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    int it = 0, sbuf = 0;
    for (int w = cluster; w < total_work; w += nclusters, ++it) {
      const TileCoord tc = decode_tile(P, w, total_work, BN, 256);
      const GemmProblemDev& pr = P.p[tc.pi];
      const EpiScalars ep{pr.bias, P.alpha, P.act, pr.N, pr.M, pr.resid, pr.ldr};
      const int buf = it & 1;
      if (!mbar_wait(&acc_full[buf], (it >> 1) & 1, ERR_EPI_WAIT)) break;
      tc_fence_after();
      const int row0 = tc.m0 + 128 * (int)crank + quarter * 32;
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + c0), v);
        if (c0 + 32 >= cend) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty_leader + buf * 8);
        }
        const int col0 = tc.n0 + c0;
        if (col0 >= ep.N) continue;
        epilogue_math(v, ep.alpha, ep, col0, lane);
        epilogue_residual(v, ep, row0 + lane, col0);
        // per-warp ring of staging chunks (8 KB): 4 bf16 or 2 fp32 chunks of 32 x 32
        const int ring = out32 ? 2 : 4;
        uint8_t* stg = stage_out + ew * STAGE_WARP_BYTES + (sbuf % ring) * (out32 ? 4096 : 2048);
        if (lane == 0) {
          if (out32) bulk_wait_read<1>();  // the chunk stored `ring` chunks ago has been read
          else bulk_wait_read<3>();
        }
        __syncwarp();
        if (out32) {
          float4* dst = reinterpret_cast<float4*>(stg + lane * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) dst[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(stg + lane * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
            dst[j ^ ((lane >> 1) & 3)] = *reinterpret_cast<uint4*>(h);
          }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0 && row0 < ep.M) {
          tma_store_3d(&pr.tc, stg, col0, row0, 0);
          bulk_commit();
        }
        ++sbuf;
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 0) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// Sum split-K partials [S][n] (stride between splits `stride`) into out, fixed order.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ out, long long n,
                                     int splits, long long stride, float beta) {
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n; i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += part[k * stride + i];
    out[i] = beta != 0.f ? beta * out[i] + s : s;
  }
}

}  // namespace maloq

// ======================================================================= host side
namespace maloq {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix (row stride ld elements),
// box {64 cols, box_rows}, 128B swizzle, zero fill out of bounds.
static const char* make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld,
                            int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return "TMA base address must be 16-byte aligned";
  if ((ld * 2) % 16 != 0) return "TMA row stride must be a multiple of 16 bytes";
  EncodeTiledFn enc = get_encode();
  if (!enc) return "cuTensorMapEncodeTiled is not available";
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? nullptr : "cuTensorMapEncodeTiled failed";
}

// Output map: 3-D {N, M, splits} over fp32 or bf16, box {32, 32, 1}; 128B swizzle for fp32
// rows (128 bytes), 64B swizzle for bf16 rows (64 bytes), matching the epilogue staging.
static const char* make_out_map(CUtensorMap* m, void* base, long long M, long long N, long long ldc, long long sstride,
                                int splits, bool fp32) {
  const int es = fp32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return "GEMM output must be 16-byte aligned";
  if ((ldc * es) % 16 != 0) return "GEMM output row stride must be a multiple of 16 bytes";
  EncodeTiledFn enc = get_encode();
  if (!enc) return "cuTensorMapEncodeTiled is not available";
  long long s2 = splits > 1 ? sstride : M * ldc;
  if (s2 <= 0) s2 = ldc;
  if ((s2 * es) % 16 != 0) return "GEMM split stride must be a multiple of 16 bytes";
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)splits};
  cuuint64_t strides[2] = {(cuuint64_t)(ldc * es), (cuuint64_t)(s2 * es)};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? nullptr : "cuTensorMapEncodeTiled (output) failed";
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
static const char* launch_t(const GemmParamsDev& P, int tiles, int splits, cudaStream_t st) {
  constexpr int smem = STAGES * (BM * BK + BN * BK) * 2 + 1024 + (2 * STAGES + 4) * 8 + 16 + 1024 + EPI_WARPS * STAGE_WARP_BYTES;
  auto k = gemm_tc_kernel<BN, STAGES, A_MN, B_MN>;
  static bool init = false;  // per process; the attribute applies to every device
  if (!init) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return "cudaFuncSetAttribute failed";
    init = true;
  }
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_sms <= 0) num_sms = 148;
  }
  const int total = tiles * splits;
  const int grid = total < num_sms ? total : num_sms;
  k<<<grid, GEMM_THREADS, smem, st>>>(P, total, tiles);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

template <int BN, int STAGES>
static const char* launch_2sm(const GemmParamsDev& P, int total, cudaStream_t st) {
  constexpr int smem = STAGES * (128 * BK + (BN / 2) * BK) * 2 + 1024 + (2 * STAGES + 4) * 8 + 16 + 1024 +
                       EPI_WARPS * STAGE_WARP_BYTES;
  auto k = gemm_tc2_kernel<BN, STAGES>;
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return "cudaFuncSetAttribute (2-SM) failed";
    init = true;
  }
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_sms <= 1) num_sms = 148;
  }
  int clusters = num_sms / 2;
  if (total < clusters) clusters = total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, P, total);
  if (e != cudaSuccess) return cudaGetErrorString(e);
  e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

const char* gemm_launch(const GemmProblem* probs, int nprob, bool a_mn, bool b_mn, bool out_fp32, int act,
                        float alpha, int splits, int bn, cudaStream_t stream) {
  if (nprob < 1 || nprob > 8) return "gemm: 1..8 problems per launch";
  if (bn != 64 && bn != 128 && bn != 256) return "gemm: bn must be 64, 128 or 256";
  if (a_mn != b_mn) return "gemm: mixed operand majors are not instantiated";
  if (splits < 1) return "gemm: splits must be >= 1";
  GemmParamsDev P;
  memset(&P, 0, sizeof(P));
  P.nprob = nprob;
  P.act = act;
  P.alpha = alpha;
  P.out_fp32 = out_fp32 ? 1 : 0;
  int tiles = 0;
  for (int i = 0; i < nprob; ++i) {
    const GemmProblem& g = probs[i];
    GemmProblemDev& d = P.p[i];
    const char* err = a_mn ? make_map(&d.ta, g.a, g.K, g.M, g.lda, BK) : make_map(&d.ta, g.a, g.M, g.K, g.lda, BM);
    if (err) return err;
    err = b_mn ? make_map(&d.tb, g.b, g.K, g.N, g.ldb, BK) : make_map(&d.tb, g.b, g.N, g.K, g.ldb, bn);
    if (err) return err;
    err = make_out_map(&d.tc, g.c, g.M, g.N, g.ldc, g.split_stride, splits, out_fp32);
    if (err) return err;
    if (g.resid != nullptr && (!out_fp32 || splits > 1)) return "gemm: a residual needs fp32 output and no split-K";
    d.c = g.c;
    d.bias = g.bias;
    d.resid = g.resid;
    d.ldr = g.ldr;
    d.ldc = g.ldc;
    d.split_stride = g.split_stride;
    d.M = g.M;
    d.N = g.N;
    d.K = g.K;
    d.tiles_n = (g.N + bn - 1) / bn;
    d.tile_begin = tiles;
    d.k_per_split = splits > 1 ? (int)(((g.K + splits - 1) / splits + BK - 1) / BK * BK) : g.K;
    tiles += ((g.M + BM - 1) / BM) * d.tiles_n;
  }
  if (tiles == 0) return nullptr;
  if (!a_mn && splits == 1 && (bn == 256 || bn == 128)) {
    // re-tile with 256-row pair tiles; the B box is BN/2 rows per CTA
    int total = 0;
    for (int i = 0; i < nprob; ++i) {
      GemmProblemDev& d = P.p[i];
      const GemmProblem& g = probs[i];
      const char* err = make_map(&d.tb, g.b, g.N, g.K, g.ldb, bn / 2);
      if (err) return err;
      d.tile_begin = total;
      total += ((g.M + 255) / 256) * d.tiles_n;
    }
    if (bn == 256) return launch_2sm<256, 4>(P, total, stream);
    return launch_2sm<128, 6>(P, total, stream);
  }
  if (!a_mn) {
    if (bn == 256) return launch_t<256, 3, false, false>(P, tiles, splits, stream);
    if (bn == 128) return launch_t<128, 4, false, false>(P, tiles, splits, stream);
    return launch_t<64, 6, false, false>(P, tiles, splits, stream);
  }
  if (bn == 256) return launch_t<256, 3, true, true>(P, tiles, splits, stream);
  if (bn == 128) return launch_t<128, 4, true, true>(P, tiles, splits, stream);
  return launch_t<64, 6, true, true>(P, tiles, splits, stream);
}

const char* gemm_splitk_reduce(const float* part, float* out, long long n, int splits, long long stride, float beta,
                               cudaStream_t stream) {
  if (n == 0) return nullptr;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(part, out, n, splits, stride, beta);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace maloq
