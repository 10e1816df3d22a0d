// Normalisation and gating kernels (CUDA cores, one pass over each row).
//
// * rms_norm_sh: degree-balanced equivariant RMS norm on rows [S, C] (S = (L+1)^2), with an
//   optional fused residual add (s = x + res; out = norm(s)).  One CTA per row, one thread
//   per channel holding the row's S coefficients; two block reductions.
//   Reference math: helm/nn/layer_norm.py:290-338.
// * layernorm_silu: silu(LayerNorm(x)) on rows of width W (<= 1024), one warp per row.
// * gate_l: the l-outer gate of the atomwise block (helm/nn/activation.py:57-77).
// * head_gate: the gated operand of the Fock head's per-degree projections
//   (helm/esen_osh.py:986-1052): row 0 the transformed scalars, every l >= 1 coefficient times
//   its activated gate (sigmoid or tanh of the raw, optionally absolute, gate, times a scale).
// Parameter gradients are written as per-CTA partial sums (grid-stride over rows) and summed
// by the caller in a fixed order, so they are deterministic.
#include "common.cuh"
#include "norm.h"
#include "head_gate.cuh"

namespace maloq {

// fp32 / bf16 element access (activations that feed a bf16 GEMM are stored as bf16)
__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

template <int L>
__device__ __forceinline__ float degree_weight(int j) {
  int l = 0;
  while ((l + 1) * (l + 1) <= j) ++l;
  return 1.f / ((2 * l + 1) * (L + 1));
}

// ------------------------------------------------------------------ rms_norm_sh
template <int L, int NW, typename TO>
__global__ void __launch_bounds__(NW * 32) rms_norm_fwd_kernel(const float* __restrict__ X,
                                                               const float* __restrict__ RES,
                                                               const float* __restrict__ aw,
                                                               const float* __restrict__ ab, TO* __restrict__ OUT,
                                                               float* __restrict__ SUM, int B, int C, float eps) {
  constexpr int S = (L + 1) * (L + 1);
  __shared__ float red[NW];
  const int c = threadIdx.x;
  const bool act = c < C;
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const size_t base = (size_t)b * S * C + c;
    float v[S];
#pragma unroll
    for (int j = 0; j < S; ++j) {
      v[j] = act ? X[base + (size_t)j * C] : 0.f;
      if (RES && act) v[j] += RES[base + (size_t)j * C];
    }
    if (SUM && act) {
#pragma unroll
      for (int j = 0; j < S; ++j) SUM[base + (size_t)j * C] = v[j];
    }
    const float mean0 = block_sum<NW>(v[0], red) / C;
    if (act) v[0] -= mean0;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < S; ++j) ss += degree_weight<L>(j) * v[j] * v[j];
    if (!act) ss = 0.f;
    const float r = rsqrtf(block_sum<NW>(ss, red) / C + eps);
    if (act) {
#pragma unroll
      for (int j = 0; j < S; ++j) {
        int l = 0;
        while ((l + 1) * (l + 1) <= j) ++l;
        float o = v[j] * r * __ldg(aw + l * C + c);
        if (j == 0) o += __ldg(ab + c);
        stf(OUT + base + (size_t)j * C, o);
      }
    }
  }
}

// G: grad of OUT; GS (optional): grad flowing into the residual sum itself.
// DX = d(sum); PART[blockIdx.x] += (d_aw [L+1, C], d_ab [C]).
template <int L, int NW, typename TG>
__global__ void __launch_bounds__(NW * 32) rms_norm_bwd_kernel(const float* __restrict__ Sx,
                                                               const TG* __restrict__ G,
                                                               const float* __restrict__ GS,
                                                               const float* __restrict__ aw, float* __restrict__ DX,
                                                               float* __restrict__ PART, int B, int C, float eps) {
  constexpr int S = (L + 1) * (L + 1);
  __shared__ float red[NW];
  const int c = threadIdx.x;
  const bool act = c < C;
  float daw[L + 1], dab = 0.f;
#pragma unroll
  for (int l = 0; l <= L; ++l) daw[l] = 0.f;
  float w[L + 1];
#pragma unroll
  for (int l = 0; l <= L; ++l) w[l] = act ? __ldg(aw + l * C + c) : 0.f;
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const size_t base = (size_t)b * S * C + c;
    float f[S], g[S];
#pragma unroll
    for (int j = 0; j < S; ++j) {
      f[j] = act ? Sx[base + (size_t)j * C] : 0.f;
      g[j] = act ? ldf(G + base + (size_t)j * C) : 0.f;
    }
    const float mean0 = block_sum<NW>(f[0], red) / C;
    if (act) f[0] -= mean0;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < S; ++j) ss += degree_weight<L>(j) * f[j] * f[j];
    if (!act) ss = 0.f;
    const float r = rsqrtf(block_sum<NW>(ss, red) / C + eps);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < S; ++j) {
      int l = 0;
      while ((l + 1) * (l + 1) <= j) ++l;
      const float gf = g[j] * w[l];
      dot += gf * f[j];
      daw[l] += g[j] * f[j] * r;
    }
    dab += g[0];
    const float D = block_sum<NW>(act ? dot : 0.f, red);
    const float k3 = r * r * r * D / C;
    float df[S];
#pragma unroll
    for (int j = 0; j < S; ++j) {
      int l = 0;
      while ((l + 1) * (l + 1) <= j) ++l;
      df[j] = r * g[j] * w[l] - k3 * degree_weight<L>(j) * f[j];
    }
    const float mdf0 = block_sum<NW>(act ? df[0] : 0.f, red) / C;
    df[0] -= mdf0;
    if (act) {
#pragma unroll
      for (int j = 0; j < S; ++j) DX[base + (size_t)j * C] = df[j] + (GS ? GS[base + (size_t)j * C] : 0.f);
    }
  }
  if (act) {
    float* p = PART + (size_t)blockIdx.x * (L + 2) * C;
#pragma unroll
    for (int l = 0; l <= L; ++l) p[l * C + c] = daw[l];
    p[(L + 1) * C + c] = dab;
  }
}

// ------------------------------------------------------------------ layernorm + silu
// One warp per row of width W (W <= 1024, VPT = ceil(W/32) values per lane).
template <int VPT>
__global__ void ln_silu_fwd_kernel(const float* __restrict__ X, const float* __restrict__ w,
                                   const float* __restrict__ b, __nv_bfloat16* __restrict__ OUT, int M, int W,
                                   float eps) {
  const int lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  for (long long row = (long long)blockIdx.x * warps + threadIdx.x / 32; row < M; row += (long long)gridDim.x * warps) {
    const float* x = X + row * W;
    float v[VPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < W ? x[c] : 0.f;
      s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
    const float mu = s / W;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      const float d = c < W ? v[i] - mu : 0.f;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffff, q, o);
    const float rs = rsqrtf(q / W + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < W) OUT[row * W + c] = __float2bfloat16_rn(silu((v[i] - mu) * rs * __ldg(w + c) + __ldg(b + c)));
    }
  }
}

template <int VPT>
__global__ void ln_silu_bwd_kernel(const float* __restrict__ X, const float* __restrict__ w,
                                   const float* __restrict__ b, const __nv_bfloat16* __restrict__ G,
                                   float* __restrict__ DX, float* __restrict__ PART, int M, int W, float eps) {
  const int lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  float dw[VPT], db[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) dw[i] = db[i] = 0.f;
  for (long long row = (long long)blockIdx.x * warps + threadIdx.x / 32; row < M; row += (long long)gridDim.x * warps) {
    const float* x = X + row * W;
    float v[VPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < W ? x[c] : 0.f;
      s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
    const float mu = s / W;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      const float d = c < W ? v[i] - mu : 0.f;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffff, q, o);
    const float rs = rsqrtf(q / W + eps);
    float xh[VPT], dxh[VPT];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      xh[i] = (v[i] - mu) * rs;
      dxh[i] = 0.f;
      if (c < W) {
        const float y = xh[i] * __ldg(w + c) + __ldg(b + c);
        const float dy = __bfloat162float(G[row * W + c]) * dsilu(y);
        dw[i] += dy * xh[i];
        db[i] += dy;
        dxh[i] = dy * __ldg(w + c);
        s1 += dxh[i];
        s2 += dxh[i] * xh[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffff, s1, o);
      s2 += __shfl_xor_sync(0xffffffff, s2, o);
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < W) DX[row * W + c] = rs * (dxh[i] - s1 / W - xh[i] * s2 / W);
    }
  }
  // per-CTA partials: [blockIdx.x][warp][2][W] summed by the caller
  float* p = PART + ((size_t)blockIdx.x * warps + threadIdx.x / 32) * 2 * W;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < W) {
      p[c] = dw[i];
      p[W + c] = db[i];
    }
  }
}

// ------------------------------------------------------------------ gate (l-outer)
// OUT[b,0,h] = silu(X[b,0,h]); OUT[b,j,h] = X[b,j,h] * tanh(g), g = Gt[b,(l_j-1)*H + h], or
// g = silu(Gt[...]) when silu_gates (Gt then holds the gate pre-activations: the SiLU of the
// atomwise block's scalar MLP is applied here instead of in a separate pass)
template <int L, typename T>
__global__ void gate_l_fwd_kernel(const T* __restrict__ X, const float* __restrict__ Gt, T* __restrict__ OUT, int B,
                                  int H, bool silu_gates) {
  constexpr int S = (L + 1) * (L + 1);
  const long long total = (long long)B * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int h = (int)(i % H);
    const long long b = i / H;
    const T* x = X + b * S * H + h;
    T* o = OUT + b * S * H + h;
    stf(o, silu(ldf(x)));
#pragma unroll
    for (int l = 1; l <= L; ++l) {
      const float g = Gt[b * L * H + (l - 1) * H + h];
      const float t = tanhf(silu_gates ? silu(g) : g);
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) stf(o + (size_t)j * H, ldf(x + (size_t)j * H) * t);
    }
  }
}

template <int L, typename T>
__global__ void gate_l_bwd_kernel(const T* __restrict__ X, const float* __restrict__ Gt, const T* __restrict__ DO,
                                  T* __restrict__ DX, float* __restrict__ DG, int B, int H, bool silu_gates) {
  constexpr int S = (L + 1) * (L + 1);
  const long long total = (long long)B * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int h = (int)(i % H);
    const long long b = i / H;
    const T* x = X + b * S * H + h;
    const T* d = DO + b * S * H + h;
    T* dx = DX + b * S * H + h;
    stf(dx, ldf(d) * dsilu(ldf(x)));
#pragma unroll
    for (int l = 1; l <= L; ++l) {
      const float g = Gt[b * L * H + (l - 1) * H + h];
      const float t = tanhf(silu_gates ? silu(g) : g);
      float acc = 0.f;
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
        const float dv = ldf(d + (size_t)j * H);
        stf(dx + (size_t)j * H, dv * t);
        acc += dv * ldf(x + (size_t)j * H);
      }
      DG[b * L * H + (l - 1) * H + h] = acc * (1.f - t * t) * (silu_gates ? dsilu(g) : 1.f);
    }
  }
}

}  // namespace maloq

// ======================================================================= host launchers
namespace maloq {

static const char* norm_err() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

#define MALOQ_L_CASE(L_, ...) \
  if (L == L_) {              \
    constexpr int LL = L_;    \
    __VA_ARGS__;              \
    return norm_err();        \
  }
#define MALOQ_DISPATCH_L(...)                                                                        \
  MALOQ_L_CASE(0, __VA_ARGS__) MALOQ_L_CASE(1, __VA_ARGS__) MALOQ_L_CASE(2, __VA_ARGS__)             \
  MALOQ_L_CASE(3, __VA_ARGS__) MALOQ_L_CASE(4, __VA_ARGS__) MALOQ_L_CASE(5, __VA_ARGS__)             \
  MALOQ_L_CASE(6, __VA_ARGS__) return "norm kernels: lmax must be 0..6";

int norm_grid(long long rows) { return (int)std::min<long long>(rows, 148 * 16); }

#define MALOQ_NW_CASES(C, ...)                                 \
  if (C <= 32) { constexpr int NWW = 1; __VA_ARGS__; }         \
  else if (C <= 64) { constexpr int NWW = 2; __VA_ARGS__; }    \
  else if (C <= 128) { constexpr int NWW = 4; __VA_ARGS__; }   \
  else if (C <= 256) { constexpr int NWW = 8; __VA_ARGS__; }   \
  else return "norm kernels: channels must be <= 256";

const char* rms_norm_fwd(int L, const float* X, const float* RES, const float* aw, const float* ab, void* OUT,
                         bool out_bf16, float* SUM, int B, int C, float eps, cudaStream_t st) {
  if (B == 0) return nullptr;
  const int grid = norm_grid(B);
  if (out_bf16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(OUT);
    MALOQ_NW_CASES(C, MALOQ_DISPATCH_L((rms_norm_fwd_kernel<LL, NWW, __nv_bfloat16><<<grid, NWW * 32, 0, st>>>(
                          X, RES, aw, ab, o, SUM, B, C, eps))))
  }
  float* o = static_cast<float*>(OUT);
  MALOQ_NW_CASES(C, MALOQ_DISPATCH_L((rms_norm_fwd_kernel<LL, NWW, float><<<grid, NWW * 32, 0, st>>>(X, RES, aw, ab, o,
                                                                                                      SUM, B, C, eps))))
}

const char* rms_norm_bwd(int L, const float* Sx, const void* G, bool g_bf16, const float* GS, const float* aw,
                         float* DX, float* PART, int B, int C, float eps, int grid, cudaStream_t st) {
  if (B == 0) return nullptr;
  if (g_bf16) {
    const __nv_bfloat16* g = static_cast<const __nv_bfloat16*>(G);
    MALOQ_NW_CASES(C, MALOQ_DISPATCH_L((rms_norm_bwd_kernel<LL, NWW, __nv_bfloat16><<<grid, NWW * 32, 0, st>>>(
                          Sx, g, GS, aw, DX, PART, B, C, eps))))
  }
  const float* g = static_cast<const float*>(G);
  MALOQ_NW_CASES(C, MALOQ_DISPATCH_L((rms_norm_bwd_kernel<LL, NWW, float><<<grid, NWW * 32, 0, st>>>(Sx, g, GS, aw, DX,
                                                                                                      PART, B, C, eps))))
}

#define MALOQ_VPT_CASES(W, ...)                                  \
  if (W <= 32) { constexpr int V = 1; __VA_ARGS__; }             \
  else if (W <= 64) { constexpr int V = 2; __VA_ARGS__; }        \
  else if (W <= 128) { constexpr int V = 4; __VA_ARGS__; }       \
  else if (W <= 256) { constexpr int V = 8; __VA_ARGS__; }       \
  else if (W <= 512) { constexpr int V = 16; __VA_ARGS__; }      \
  else if (W <= 1024) { constexpr int V = 32; __VA_ARGS__; }     \
  else return "layernorm: width must be <= 1024";

const char* ln_silu_fwd(const float* X, const float* w, const float* b, __nv_bfloat16* OUT, int M, int W, float eps,
                        cudaStream_t st) {
  if (M == 0) return nullptr;
  const int grid = (int)std::min<long long>((M + 7) / 8, 148 * 16);
  MALOQ_VPT_CASES(W, (ln_silu_fwd_kernel<V><<<grid, 256, 0, st>>>(X, w, b, OUT, M, W, eps)))
  return norm_err();
}

const char* ln_silu_bwd(const float* X, const float* w, const float* b, const __nv_bfloat16* G, float* DX, float* PART,
                        int M, int W, float eps, int grid, cudaStream_t st) {
  if (M == 0) return nullptr;
  MALOQ_VPT_CASES(W, (ln_silu_bwd_kernel<V><<<grid, 256, 0, st>>>(X, w, b, G, DX, PART, M, W, eps)))
  return norm_err();
}

const char* gate_l_fwd(int L, const void* X, const float* Gt, void* OUT, bool bf16, int B, int H, cudaStream_t st,
                       bool silu_gates) {
  if (B == 0) return nullptr;
  const int grid = (int)std::min<long long>(((long long)B * H + 255) / 256, 148 * 32);
  if (bf16) {
    MALOQ_DISPATCH_L((gate_l_fwd_kernel<LL, __nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(X), Gt, static_cast<__nv_bfloat16*>(OUT), B, H, silu_gates)))
  }
  MALOQ_DISPATCH_L((gate_l_fwd_kernel<LL, float><<<grid, 256, 0, st>>>(static_cast<const float*>(X), Gt,
                                                                      static_cast<float*>(OUT), B, H, silu_gates)))
}

const char* gate_l_bwd(int L, const void* X, const float* Gt, const void* DO, void* DX, float* DG, bool bf16, int B,
                       int H, cudaStream_t st, bool silu_gates) {
  if (B == 0) return nullptr;
  const int grid = (int)std::min<long long>(((long long)B * H + 255) / 256, 148 * 32);
  if (bf16) {
    MALOQ_DISPATCH_L((gate_l_bwd_kernel<LL, __nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(X), Gt, static_cast<const __nv_bfloat16*>(DO),
        static_cast<__nv_bfloat16*>(DX), DG, B, H, silu_gates)))
  }
  MALOQ_DISPATCH_L((gate_l_bwd_kernel<LL, float><<<grid, 256, 0, st>>>(static_cast<const float*>(X), Gt,
                                                                      static_cast<const float*>(DO),
                                                                      static_cast<float*>(DX), DG, B, H, silu_gates)))
}

const char* head_gate_fwd(int L, const float* X, const float* SV, __nv_bfloat16* A, int act, float scale, bool absg,
                          int B, int C, cudaStream_t st) {
  if (B == 0) return nullptr;
  const int grid = (int)std::min<long long>(((long long)B * C + 255) / 256, 148 * 32);
  if (act == 0) {
    MALOQ_DISPATCH_L((head_gate_fwd_kernel<LL, 0><<<grid, 256, 0, st>>>(X, SV, A, B, C, scale, absg)))
  }
  MALOQ_DISPATCH_L((head_gate_fwd_kernel<LL, 1><<<grid, 256, 0, st>>>(X, SV, A, B, C, scale, absg)))
}

const char* head_gate_bwd(int L, const float* X, const float* SV, const float* DA, float* DX, float* DSV, int act,
                          float scale, bool absg, int B, int C, cudaStream_t st) {
  if (B == 0) return nullptr;
  const int grid = (int)std::min<long long>(((long long)B * C + 255) / 256, 148 * 32);
  if (act == 0) {
    MALOQ_DISPATCH_L((head_gate_bwd_kernel<LL, 0><<<grid, 256, 0, st>>>(X, SV, DA, DX, DSV, B, C, scale, absg)))
  }
  MALOQ_DISPATCH_L((head_gate_bwd_kernel<LL, 1><<<grid, 256, 0, st>>>(X, SV, DA, DX, DSV, B, C, scale, absg)))
}

}  // namespace maloq
