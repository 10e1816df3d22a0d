// Grouped bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   C[p] (M x N) = alpha * A[p] (M x K) * B[p]^T (K x N) (+ bias[N]) (act)
//
// A and B are bf16 and either K-major (row-major [M,K] / [N,K]) or MN-major (row-major
// [K,M] / [K,N], used for weight gradients where K is the edge dimension).  Up to eight
// problems run in one launch (the per-|m| SO(2) GEMMs of a layer).  Optional split-K
// writes fp32 partials [split][M][N]; gemm_splitk_reduce sums them in a fixed order, so
// weight gradients are deterministic.
//
// CTA = 128 threads, tile 128 x BN x 64, STAGES-deep TMA ring:
//   warp 0 (one elected lane): TMA producer        - waits "empty", loads the A/B tiles
//   warp 1 (one elected lane): tcgen05.mma issuer  - waits "full", 4 MMAs (K=16), commits "empty"
//   all 4 warps: epilogue - tcgen05.ld of TMEM lanes 32w..32w+31, bias/activation, store.
// Accumulators live in TMEM (BN fp32 columns x 128 lanes).  TMA loads use no multicast.
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm.h"

namespace maloq {

constexpr int BM = 128;
constexpr int BK = 64;

struct alignas(64) GemmProblemDev {
  CUtensorMap ta;
  CUtensorMap tb;
  void* c;
  const float* bias;
  long long ldc;
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

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(128, 1) gemm_tc_kernel(const __grid_constant__ GemmParamsDev P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  int t = blockIdx.x, pi = 0;
#pragma unroll 1
  for (int q = 1; q < P.nprob; ++q)
    if (t >= P.p[q].tile_begin) pi = q;
  const GemmProblemDev& pr = P.p[pi];
  t -= pr.tile_begin;
  const int m0 = (t / pr.tiles_n) * BM;
  const int n0 = (t % pr.tiles_n) * BN;
  const int split = blockIdx.y;
  const int k_begin = split * pr.k_per_split;
  const int k_end = min(pr.K, k_begin + pr.k_per_split);
  const int k_tiles = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, BN < 32 ? 32 : BN);
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&pr.ta);
    prefetch_tmap(&pr.tb);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % STAGES;
        if (kt >= STAGES && !mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1, ERR_TMA_WAIT)) break;
        mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
        const int k = k_begin + kt * BK;
        uint8_t* a = sA + s * A_BYTES;
        uint8_t* b = sB + s * B_BYTES;
        if constexpr (A_MN) {
          tma_load_2d(a, &pr.ta, &full[s], m0, k);
          tma_load_2d(a + BK * 128, &pr.ta, &full[s], m0 + 64, k);
        } else {
          tma_load_2d(a, &pr.ta, &full[s], k, m0);
        }
        if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * BK * 128, &pr.tb, &full[s], n0 + 64 * j, k);
        } else {
          tma_load_2d(b, &pr.tb, &full[s], k, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      bool ok = true;
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % STAGES;
        if (!mbar_wait(&full[s], (kt / STAGES) & 1, ERR_MMA_WAIT)) {
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
          umma_f16(tmem, ad, bd, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(done);
    }
  }
  __syncwarp();

  // ---------------- epilogue (all 4 warps; tcgen05.ld is warp-collective)
  const int row = m0 + warp * 32 + lane;
  const bool have = k_tiles > 0 && mbar_wait(done, 0, ERR_EPI_WAIT);
  tc_fence_after();
  char* cbase = reinterpret_cast<char*>(pr.c);
  const size_t esz = P.out_fp32 ? 4 : 2;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    float v[32];
    if (have) {
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
    const int col0 = n0 + c0;
    if (row >= pr.M || col0 >= pr.N) continue;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = v[j] * P.alpha;
      if (pr.bias != nullptr && col0 + j < pr.N) x += __ldg(pr.bias + col0 + j);
      if (P.act == 1) x = silu(x);
      v[j] = x;
    }
    char* rowp = cbase + ((size_t)split * pr.split_stride + (size_t)row * pr.ldc + col0) * esz;
    const bool full_chunk = col0 + 32 <= pr.N && ((reinterpret_cast<uintptr_t>(rowp) & 15) == 0);
    if (P.out_fp32) {
      float* o = reinterpret_cast<float*>(rowp);
      if (full_chunk) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < 32 && col0 + j < pr.N; ++j) o[j] = v[j];
      }
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(rowp);
      if (full_chunk) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          __nv_bfloat162 h[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[j + 2 * q], v[j + 2 * q + 1]);
          *reinterpret_cast<uint4*>(o + j) = *reinterpret_cast<uint4*>(h);
        }
      } else {
        for (int j = 0; j < 32 && col0 + j < pr.N; ++j) o[j] = __float2bfloat16_rn(v[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, BN < 32 ? 32 : BN);
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

template <int BN, int STAGES, bool A_MN, bool B_MN>
static const char* launch_t(const GemmParamsDev& P, int tiles, int splits, cudaStream_t st) {
  constexpr int smem = STAGES * (BM * BK + BN * BK) * 2 + 1024 + (2 * STAGES + 1) * 8 + 16;
  auto k = gemm_tc_kernel<BN, STAGES, A_MN, B_MN>;
  static bool init = false;  // per process; the attribute applies to every device
  if (!init) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return "cudaFuncSetAttribute failed";
    init = true;
  }
  k<<<dim3(tiles, splits), 128, smem, st>>>(P);
  cudaError_t e = cudaGetLastError();
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
    d.c = g.c;
    d.bias = g.bias;
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
  if (!a_mn) {
    if (bn == 256) return launch_t<256, 3, false, false>(P, tiles, splits, stream);
    if (bn == 128) return launch_t<128, 5, false, false>(P, tiles, splits, stream);
    return launch_t<64, 6, false, false>(P, tiles, splits, stream);
  }
  if (bn == 256) return launch_t<256, 3, true, true>(P, tiles, splits, stream);
  if (bn == 128) return launch_t<128, 5, true, true>(P, tiles, splits, stream);
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
