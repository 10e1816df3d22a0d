// Edge-frame kernels of the Edgewise message pass (CUDA cores; memory-bound).
//
// Layouts: node features X [N, S, C] fp32 (S = (L+1)^2 l-major coefficients), edge
// embeddings XE [E, S, C] fp32, rotation ROT [E, R, S] fp32 (R m-major rows, |m| <= mmax;
// row k only has entries in the 2l+1 columns of its degree), messages A / H / Y
// [E, R*Cm] bf16 (row k of edge e at columns k*Cm .. k*Cm+Cm-1), radial modulation
// RAD [E, NS*Cin] fp32 (NS slots, see edge_frame.cuh).
// Edges are sorted by destination; dst_ptr [N+1] gives each node's incoming-edge range and
// src_perm/src_ptr the same for sources, so every reduction over edges is a fixed-order
// segmented sum (deterministic, no atomics).
// Kernels are templated on the frame (L, MM) so the row/degree structure is compile-time.
#include "common.cuh"
#include "edge.h"
#include "edge_frame.cuh"

namespace maloq {

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }

// Source rows of the gather: local rows s < n_own come from X; with a halo (peers != nullptr)
// rows s >= n_own are halo node h = s - n_own, read from the owner's staging buffer
// peers[halo_owner[h]] at row halo_row[h] - a load over NVLink.
struct HaloRef {
  const float* const* peers;
  const int* halo_owner;
  const long long* halo_row;
  long long n_own;
  long long n_src, n_dst;  // valid source / destination rows (bounds checks)
  // backward with recv != nullptr: the gradient row of halo node h (row n_own + h) is stored
  // straight into slot recv_slot[h] of its owner's receive buffer recv[halo_owner[h]] (a store
  // over NVLink) instead of into DX
  float* const* recv;
  const long long* recv_slot;
};

__device__ __forceinline__ const float* src_row(const float* X, long long s, int S, int C, const HaloRef& H) {
  if (H.peers == nullptr || s < H.n_own) return X + s * S * C;
  const long long h = s - H.n_own;
  return H.peers[H.halo_owner[h]] + H.halo_row[h] * S * C;
}

// ---------------------------------------------------------------- gather + rotate + modulate
// A[e, k, c'] = rad[e, slot(k)*Cin + c'] * sum_{j in degree l_k} rot[e,k,j] * in[e, j, c']
// in = [X[src] | X[dst] | XE[e]] along channels (Cin = 2C or 3C); rad is bf16.
// Edge-parallel: Q edge lanes per CTA, two adjacent channels per thread (C even).
template <int S>
struct EdgeLanes {
  static constexpr int Q = S <= 25 ? 4 : 2;
};

template <int L, int MM>
__global__ void __launch_bounds__(256) gather_rotate_fwd_kernel(
    const float* __restrict__ X, const float* __restrict__ XE, const long long* __restrict__ src,
    const long long* __restrict__ dst, const float* __restrict__ rot, const __nv_bfloat16* __restrict__ rad,
    __nv_bfloat16* __restrict__ A, int E, int C, int Cin, const HaloRef H) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R, Q = EdgeLanes<S>::Q;
  const int cpair = threadIdx.x % 64, q = threadIdx.x / 64;
  const long long e = (long long)blockIdx.x * Q + q;
  const int cp = 2 * (blockIdx.y * 64 + cpair);
  if (e >= E || cp >= Cin) return;
  if (!MALOQ_IN_BOUNDS(src[e] >= 0 && src[e] < H.n_src && dst[e] >= 0 && dst[e] < H.n_dst)) return;
  const float* base;
  if (cp < C) base = src_row(X, src[e], S, C, H) + cp;
  else if (cp < 2 * C) base = X + (size_t)dst[e] * S * C + (cp - C);
  else base = XE + (size_t)e * S * C + (cp - 2 * C);
  float2 in[S];
#pragma unroll
  for (int j = 0; j < S; ++j) in[j] = __ldg(reinterpret_cast<const float2*>(base + (size_t)j * C));
  const float* re = rot + (size_t)e * R * S;
  const __nv_bfloat16* rd = rad ? rad + (size_t)e * F::NS * Cin + cp : nullptr;
  __nv_bfloat16* out = A + (size_t)e * R * Cin + cp;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int l = F::row_l(k);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
      const float r = __ldg(re + k * S + j);
      acc.x += r * in[j].x;
      acc.y += r * in[j].y;
    }
    if (rd) {
      const float2 m = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(rd + (size_t)F::slot(k) * Cin));
      acc.x *= m.x;
      acc.y *= m.y;
    }
    *reinterpret_cast<__nv_bfloat162*>(out + (size_t)k * Cin) = __floats2bfloat162_rn(acc.x, acc.y);
  }
}

// V adjacent channels (V = 1 or 2) loaded to / stored from fp32 registers v[0..V).
template <int V>
__device__ __forceinline__ void ldv(float* v, const float* p) {
  if constexpr (V == 2) {
    const float2 t = __ldg(reinterpret_cast<const float2*>(p));
    v[0] = t.x;
    v[1] = t.y;
  } else {
    v[0] = __ldg(p);
  }
}
template <int V>
__device__ __forceinline__ void ldv(float* v, const __nv_bfloat16* p) {
  if constexpr (V == 2) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = t.x;
    v[1] = t.y;
  } else {
    v[0] = __bfloat162float(*p);
  }
}
template <int V>
__device__ __forceinline__ void stv(float* p, const float* v) {
  if constexpr (V == 2) *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  else *p = v[0];
}
template <int V>
__device__ __forceinline__ void stv(__nv_bfloat16* p, const float* v) {
  if constexpr (V == 2) *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  else *p = __float2bfloat16_rn(v[0]);
}

// One m-major row K (and its -m partner) of the backward of gather_rotate, with the frame's
// row structure folded at compile time (template recursion over K).
template <int L, int MM, int V, int K>
__device__ __forceinline__ void gather_rotate_bwd_rows(const float* __restrict__ re, const float* g, const float* r,
                                                       bool has_rad, __nv_bfloat16* __restrict__ drd, int Cin,
                                                       const float* in, float* din) {
  using F = Frame<L, MM>;
  constexpr int S = F::S;
  if constexpr (K < F::R) {
    if constexpr (F::leads(K)) {
      constexpr int KP = F::pair(K), l = F::row_l(K), SL = F::slot(K);
      constexpr int NQ = KP < 0 ? 1 : 2;
      float dr[V];
#pragma unroll
      for (int i = 0; i < V; ++i) dr[i] = 0.f;
#pragma unroll
      for (int qq = 0; qq < NQ; ++qq) {
        const int kk = qq == 0 ? K : KP;
#pragma unroll
        for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
          const float rv = __ldg(re + kk * S + j);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const float gk = g[kk * V + i];
            dr[i] += gk * rv * in[j * V + i];
            din[j * V + i] += rv * (gk * r[SL * V + i]);
          }
        }
      }
      if (has_rad) stv<V>(drd + (size_t)SL * Cin, dr);
    }
    gather_rotate_bwd_rows<L, MM, V, K + 1>(re, g, r, has_rad, drd, Cin, in, din);
  }
}

// One edge's contribution to the backward of gather_rotate for V channels at offset `off` of
// the Cin channels (in/din: [S][V] registers): u = rot . in (recomputed), dU = dA * rad,
// dRAD[slot] = sum over the slot's rows of dA * u (written), din += rot^T dU.
template <int L, int MM, int V>
__device__ __forceinline__ void gather_rotate_bwd_edge(const float* __restrict__ re, const __nv_bfloat16* __restrict__ ga,
                                                       const __nv_bfloat16* __restrict__ rd,
                                                       __nv_bfloat16* __restrict__ drd, int Cin, const float* in,
                                                       float* din) {
  using F = Frame<L, MM>;
  constexpr int R = F::R;
  float g[R * V], r[F::NS * V];
#pragma unroll
  for (int k = 0; k < R; ++k) ldv<V>(g + k * V, ga + (size_t)k * Cin);
#pragma unroll
  for (int sl = 0; sl < F::NS; ++sl) {
    if (rd) ldv<V>(r + sl * V, rd + (size_t)sl * Cin);
    else
#pragma unroll
      for (int i = 0; i < V; ++i) r[sl * V + i] = 1.f;
  }
  gather_rotate_bwd_rows<L, MM, V, 0>(re, g, r, rd != nullptr, drd, Cin, in, din);
}

// Node gradients of gather_rotate, one CTA per (node n of the source space, 64*V channels):
// DX[n] = sum over n's incoming edges of the x[dst] part (channels C..2C) + sum over n's
// outgoing edges (src CSR) of the x[src] part (channels 0..C), both recomputed from dA in a
// fixed order (Q edge lanes of 64 threads, lane sums combined in shared memory) - no per-edge
// gradient rows are stored.  Both parts use the node's own row X[n] (a peer row for halo
// nodes).  The radial gradient DRAD of those channels is written per edge on the way.
template <int L, int MM, int V, int Q>
__global__ void __launch_bounds__(64 * Q) gather_rotate_bwd_nodes_kernel(
    const float* __restrict__ X, const float* __restrict__ rot, const __nv_bfloat16* __restrict__ rad,
    const __nv_bfloat16* __restrict__ dA, const long long* __restrict__ dst_ptr,
    const long long* __restrict__ src_perm, const long long* __restrict__ src_ptr, float* __restrict__ DX,
    __nv_bfloat16* __restrict__ DRAD, int N, int C, int Cin, long long E, const HaloRef H) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R;
  constexpr int LIST = 256;  // edge ids staged in shared memory per CTA
  extern __shared__ float red_s[];  // [Q-1][S][64*V]
  __shared__ long long elist[LIST];
  const int n = blockIdx.x;
  const int t = threadIdx.x % 64, q = threadIdx.x / 64;
  const int c = V * (blockIdx.y * 64 + t);
  const bool active = c < C;
  const long long d0 = dst_ptr[n], nd = dst_ptr[n + 1] - d0;
  const long long s0 = src_ptr[n], ns = src_ptr[n + 1] - s0;
  const long long total = nd + ns;
  // the node's edges: incoming (x[dst] part) then outgoing (x[src] part, through src_perm)
  for (long long i = threadIdx.x; i < total && i < LIST; i += blockDim.x)
    elist[i] = i < nd ? d0 + i : src_perm[s0 + i - nd];
  __syncthreads();
  float din[S * V];
#pragma unroll
  for (int j = 0; j < S * V; ++j) din[j] = 0.f;
  if (active) {
    float in[S * V];
    const float* xr = src_row(X, n, S, C, H) + c;
#pragma unroll
    for (int j = 0; j < S; ++j) ldv<V>(in + j * V, xr + (size_t)j * C);
#pragma unroll 1
    for (long long i = q; i < total; i += Q) {
      const long long e = i < LIST ? elist[i] : (i < nd ? d0 + i : src_perm[s0 + i - nd]);
      const int off = i < nd ? C : 0;
      if (!MALOQ_IN_BOUNDS(e >= 0 && e < E)) continue;
      const size_t eo = (size_t)e * F::NS * Cin + off + c;
      gather_rotate_bwd_edge<L, MM, V>(rot + (size_t)e * R * S, dA + (size_t)e * R * Cin + off + c,
                                       rad ? rad + eo : nullptr, DRAD ? DRAD + eo : nullptr, Cin, in, din);
    }
  }
  if (q > 0) {
#pragma unroll
    for (int j = 0; j < S; ++j)
#pragma unroll
      for (int i = 0; i < V; ++i) red_s[((q - 1) * S + j) * 64 * V + i * 64 + t] = din[j * V + i];
  }
  __syncthreads();
  if (q > 0 || !active) return;
#pragma unroll
  for (int p = 0; p < Q - 1; ++p)
#pragma unroll
    for (int j = 0; j < S; ++j)
#pragma unroll
      for (int i = 0; i < V; ++i) din[j * V + i] += red_s[(p * S + j) * 64 * V + i * 64 + t];
  float* o = DX + (size_t)n * S * C + c;
  if (H.recv != nullptr && n >= H.n_own) {  // a halo node: straight into its owner's receive slot
    const long long h = n - H.n_own;
    o = H.recv[H.halo_owner[h]] + (size_t)H.recv_slot[h] * S * C + c;
  }
#pragma unroll
  for (int j = 0; j < S; ++j) stv<V>(o + (size_t)j * C, din + j * V);
}

// Edge-embedding part of the gather_rotate backward (Cin = 3C): DXE[e] (channels 2C..3C) and
// those channels of DRAD, edge-parallel.
template <int L, int MM>
__global__ void __launch_bounds__(256) gather_rotate_bwd_edges_kernel(
    const float* __restrict__ XE, const float* __restrict__ rot, const __nv_bfloat16* __restrict__ rad,
    const __nv_bfloat16* __restrict__ dA, float* __restrict__ DXE, __nv_bfloat16* __restrict__ DRAD, int E, int C,
    int Cin) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R, Q = EdgeLanes<S>::Q;
  const int cpair = threadIdx.x % 64, q = threadIdx.x / 64;
  const long long e = (long long)blockIdx.x * Q + q;
  const int c = 2 * (blockIdx.y * 64 + cpair);
  if (e >= E || c >= C) return;
  float in[S * 2], din[S * 2];
  const float* xr = XE + (size_t)e * S * C + c;
#pragma unroll
  for (int j = 0; j < S; ++j) {
    ldv<2>(in + 2 * j, xr + (size_t)j * C);
    din[2 * j] = din[2 * j + 1] = 0.f;
  }
  const size_t eo = (size_t)e * F::NS * Cin + 2 * C + c;
  gather_rotate_bwd_edge<L, MM, 2>(rot + (size_t)e * R * S, dA + (size_t)e * R * Cin + 2 * C + c,
                                   rad ? rad + eo : nullptr, DRAD ? DRAD + eo : nullptr, Cin, in, din);
  float* o = DXE + (size_t)e * S * C + c;
#pragma unroll
  for (int j = 0; j < S; ++j) stv<2>(o + (size_t)j * C, din + 2 * j);
}

// DX[n] = sum_{e: dst=n} DDST[e] + sum_{e: src=n} DSRC[e], both in fixed (CSR) order.
__global__ void node_reduce_kernel(const float* __restrict__ DDST, const long long* __restrict__ dst_ptr,
                                   const float* __restrict__ DSRC, const long long* __restrict__ src_perm,
                                   const long long* __restrict__ src_ptr, float* __restrict__ DX, int N, int SC,
                                   long long n_dst_rows, long long n_src_rows) {
  const int n = blockIdx.x;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;
  if (n >= N || i >= SC) return;
  float s = 0.f;
  if (DDST) {
    if (!MALOQ_IN_BOUNDS(dst_ptr[n] >= 0 && dst_ptr[n + 1] <= n_dst_rows)) return;
    for (long long e = dst_ptr[n]; e < dst_ptr[n + 1]; ++e) s += DDST[(size_t)e * SC + i];
  }
  if (DSRC)
    for (long long q = src_ptr[n]; q < src_ptr[n + 1]; ++q) {
      if (!MALOQ_IN_BOUNDS(src_perm[q] >= 0 && src_perm[q] < n_src_rows)) return;
      s += DSRC[(size_t)src_perm[q] * SC + i];
    }
  DX[(size_t)n * SC + i] = s;
}

// Halo gradient push: row h of G (halo rows of the extended-space gradient) is stored into
// slot recv_slot[h] of its owner's receive buffer recv[halo_owner[h]] (a store over NVLink).
__global__ void halo_push_kernel(const float* __restrict__ G, float* const* __restrict__ recv,
                                 const int* __restrict__ halo_owner, const long long* __restrict__ recv_slot,
                                 long long n_halo, int SC) {
  const long long h = blockIdx.x;
  if (h >= n_halo) return;
  const float4* src = reinterpret_cast<const float4*>(G + h * SC);
  float4* dst = reinterpret_cast<float4*>(recv[halo_owner[h]] + recv_slot[h] * SC);
  for (int i = threadIdx.x; i < SC / 4; i += blockDim.x) dst[i] = src[i];
}

// Halo rows copied out of their owners' staging slots (peer loads over NVLink):
// OUT[h, :] = peers[halo_owner[h]][halo_row[h] * SC + :]
__global__ void halo_fetch_kernel(const float* const* __restrict__ peers, const int* __restrict__ halo_owner,
                                  const long long* __restrict__ halo_row, float* __restrict__ OUT, long long n_halo,
                                  int SC) {
  const long long h = blockIdx.x;
  if (h >= n_halo) return;
  const float4* src = reinterpret_cast<const float4*>(peers[halo_owner[h]] + halo_row[h] * SC);
  float4* dst = reinterpret_cast<float4*>(OUT + h * SC);
  for (int i = threadIdx.x; i < SC / 4; i += blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------- rotate back
// Node path: OUT[n, j, c] = scale * sum_{e: dst=n} sum_{k<Rk} rot[e,k,j] Y[e, koff + k*C + c] (+ BASE)
template <int L, int MM>
__global__ void __launch_bounds__(128) rotate_back_scatter_kernel(
    const __nv_bfloat16* __restrict__ Y, int ldy, int koff, const float* __restrict__ rot,
    const long long* __restrict__ dst_ptr, const float* __restrict__ base, float* __restrict__ out, int N, int C,
    int Rk, float scale) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R;
  const int n = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (n >= N || c >= C) return;
  float acc[S];
#pragma unroll
  for (int j = 0; j < S; ++j) acc[j] = 0.f;
#pragma unroll 1
  for (long long e = dst_ptr[n]; e < dst_ptr[n + 1]; ++e) {
    const float* re = rot + (size_t)e * R * S;
    const __nv_bfloat16* ye = Y + (size_t)e * ldy + koff + c;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (k >= Rk) break;
      const int l = F::row_l(k);
      const float y = bf2f(ye[(size_t)k * C]);
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) acc[j] += __ldg(re + k * S + j) * y;
    }
  }
  float* o = out + (size_t)n * S * C + c;
  const float* b = base ? base + (size_t)n * S * C + c : nullptr;
#pragma unroll
  for (int j = 0; j < S; ++j) o[(size_t)j * C] = acc[j] * scale + (b ? b[(size_t)j * C] : 0.f);
}

// Edge path: OUT[e, j, c] = sum_{k<Rk} rot[e,k,j] Y[e, koff + k*C + c]
template <int L, int MM>
__global__ void __launch_bounds__(128) rotate_back_edge_kernel(const __nv_bfloat16* __restrict__ Y, int ldy, int koff,
                                                               const float* __restrict__ rot, float* __restrict__ out,
                                                               int E, int C, int Rk) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R;
  const int e = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= E || c >= C) return;
  float acc[S];
#pragma unroll
  for (int j = 0; j < S; ++j) acc[j] = 0.f;
  const float* re = rot + (size_t)e * R * S;
  const __nv_bfloat16* ye = Y + (size_t)e * ldy + koff + c;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (k >= Rk) break;
    const int l = F::row_l(k);
    const float y = bf2f(ye[(size_t)k * C]);
#pragma unroll
    for (int j = l * l; j < (l + 1) * (l + 1); ++j) acc[j] += __ldg(re + k * S + j) * y;
  }
  float* o = out + (size_t)e * S * C + c;
#pragma unroll
  for (int j = 0; j < S; ++j) o[(size_t)j * C] = acc[j];
}

// Backward of both rotate-back kernels: DY[e, k*C + c] = scale * sum_j rot[e,k,j] G[row(e), j, c],
// row(e) = dst[e] (node path) or e (edge path); bf16 (DY) and/or fp32 (DYf) output.
template <int L, int MM>
__global__ void __launch_bounds__(128) rotate_grad_kernel(const float* __restrict__ G,
                                                          const long long* __restrict__ rows,
                                                          const float* __restrict__ rot, __nv_bfloat16* __restrict__ DY,
                                                          float* __restrict__ DYf, int E, int C, int Rk, float scale) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R;
  const int e = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= E || c >= C) return;
  const long long r = rows ? rows[e] : e;
  float g[S];
#pragma unroll
  for (int j = 0; j < S; ++j) g[j] = __ldg(G + ((size_t)r * S + j) * C + c);
  const float* re = rot + (size_t)e * R * S;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (k >= Rk) break;
    const int l = F::row_l(k);
    float acc = 0.f;
#pragma unroll
    for (int j = l * l; j < (l + 1) * (l + 1); ++j) acc += __ldg(re + k * S + j) * g[j];
    acc *= scale;
    if (DY) DY[((size_t)e * Rk + k) * C + c] = __float2bfloat16_rn(acc);
    if (DYf) DYf[((size_t)e * Rk + k) * C + c] = acc;
  }
}

// ---------------------------------------------------------------- rotate back, channel pairs
// The same three maps with two adjacent channels per thread (bf16x2 / float2 accesses, two FMAs
// per rotation entry) and Q edges in flight per CTA (Q "edge lanes" of 64 channel pairs).  Used
// when C, ldy and koff are even.  Node paths walk a destination's edges through its CSR range;
// the lanes' partial sums are combined in shared memory in a fixed order (deterministic).
template <int L, int MM>
__global__ void __launch_bounds__(256) rotate_back_scatter2_kernel(
    const __nv_bfloat16* __restrict__ Y, int ldy, int koff, const float* __restrict__ rot,
    const long long* __restrict__ dst_ptr, const float* __restrict__ base, float* __restrict__ out, int N, int C,
    int Rk, float scale) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R, Q = EdgeLanes<S>::Q;
  extern __shared__ float2 red2[];  // [Q-1][S][64]
  const int n = blockIdx.x;
  const int cp = threadIdx.x % 64, q = threadIdx.x / 64;
  const int c = 2 * (blockIdx.y * 64 + cp);
  const bool active = c < C;
  float2 acc[S];
#pragma unroll
  for (int j = 0; j < S; ++j) acc[j] = make_float2(0.f, 0.f);
  if (active) {
#pragma unroll 1
    for (long long e = dst_ptr[n] + q; e < dst_ptr[n + 1]; e += Q) {
      const float* re = rot + (size_t)e * R * S;
      const __nv_bfloat16* ye = Y + (size_t)e * ldy + koff + c;
#pragma unroll
      for (int k = 0; k < R; ++k) {
        if (k >= Rk) break;
        const int l = F::row_l(k);
        const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(ye + (size_t)k * C));
#pragma unroll
        for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
          const float r = __ldg(re + k * S + j);
          acc[j].x += r * y.x;
          acc[j].y += r * y.y;
        }
      }
    }
  }
  if (q > 0) {
#pragma unroll
    for (int j = 0; j < S; ++j) red2[((q - 1) * S + j) * 64 + cp] = acc[j];
  }
  __syncthreads();
  if (q > 0 || !active) return;
#pragma unroll
  for (int p = 0; p < Q - 1; ++p)
#pragma unroll
    for (int j = 0; j < S; ++j) {
      const float2 v = red2[(p * S + j) * 64 + cp];
      acc[j].x += v.x;
      acc[j].y += v.y;
    }
  float* o = out + (size_t)n * S * C + c;
  const float* b = base ? base + (size_t)n * S * C + c : nullptr;
#pragma unroll
  for (int j = 0; j < S; ++j) {
    float2 v = make_float2(acc[j].x * scale, acc[j].y * scale);
    if (b) {
      const float2 bv = *reinterpret_cast<const float2*>(b + (size_t)j * C);
      v.x += bv.x;
      v.y += bv.y;
    }
    *reinterpret_cast<float2*>(o + (size_t)j * C) = v;
  }
}

template <int L, int MM>
__global__ void __launch_bounds__(256) rotate_back_edge2_kernel(const __nv_bfloat16* __restrict__ Y, int ldy,
                                                                int koff, const float* __restrict__ rot,
                                                                float* __restrict__ out, int E, int C, int Rk) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R, Q = EdgeLanes<S>::Q;
  const int cp = threadIdx.x % 64, q = threadIdx.x / 64;
  const long long e = (long long)blockIdx.x * Q + q;
  const int c = 2 * (blockIdx.y * 64 + cp);
  if (e >= E || c >= C) return;
  float2 acc[S];
#pragma unroll
  for (int j = 0; j < S; ++j) acc[j] = make_float2(0.f, 0.f);
  const float* re = rot + (size_t)e * R * S;
  const __nv_bfloat16* ye = Y + (size_t)e * ldy + koff + c;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (k >= Rk) break;
    const int l = F::row_l(k);
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(ye + (size_t)k * C));
#pragma unroll
    for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
      const float r = __ldg(re + k * S + j);
      acc[j].x += r * y.x;
      acc[j].y += r * y.y;
    }
  }
  float* o = out + (size_t)e * S * C + c;
#pragma unroll
  for (int j = 0; j < S; ++j) *reinterpret_cast<float2*>(o + (size_t)j * C) = acc[j];
}

// DY[e, k*C + c] = scale * sum_j rot[e,k,j] G[row, j, c], edge-parallel (NODE = false): row = e,
// or out_ptr[e] when given (the node path: each edge's destination row).  NODE = true walks a
// destination's edge range instead (G[n] loaded once per lane); it leaves too few CTAs at
// molecular node counts and is not launched.
template <int L, int MM, bool NODE>
__global__ void __launch_bounds__(256) rotate_grad2_kernel(const float* __restrict__ G,
                                                           const long long* __restrict__ out_ptr,
                                                           const float* __restrict__ rot,
                                                           __nv_bfloat16* __restrict__ DY, float* __restrict__ DYf,
                                                           int rows, int C, int Rk, float scale) {
  using F = Frame<L, MM>;
  constexpr int S = F::S, R = F::R, Q = EdgeLanes<S>::Q;
  const int cp = threadIdx.x % 64, q = threadIdx.x / 64;
  const int c = 2 * (blockIdx.y * 64 + cp);
  long long r, e0, e1;
  if (NODE) {
    r = blockIdx.x;
    e0 = out_ptr[r] + q;
    e1 = out_ptr[r + 1];
  } else {
    e0 = (long long)blockIdx.x * Q + q;
    e1 = e0 + 1;
    if (e0 >= rows || c >= C) return;
    r = out_ptr ? out_ptr[e0] : e0;  // edge path: out_ptr (if given) is the edge's gradient row
  }
  if ((NODE && r >= rows) || c >= C) return;
  float2 g[S];
#pragma unroll
  for (int j = 0; j < S; ++j) g[j] = __ldg(reinterpret_cast<const float2*>(G + ((size_t)r * S + j) * C + c));
#pragma unroll 1
  for (long long e = e0; e < e1; e += (NODE ? Q : 1)) {
    const float* re = rot + (size_t)e * R * S;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (k >= Rk) break;
      const int l = F::row_l(k);
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = l * l; j < (l + 1) * (l + 1); ++j) {
        const float rv = __ldg(re + k * S + j);
        acc.x += rv * g[j].x;
        acc.y += rv * g[j].y;
      }
      acc.x *= scale;
      acc.y *= scale;
      const size_t o = ((size_t)e * Rk + k) * C + c;
      if (DY) *reinterpret_cast<__nv_bfloat162*>(DY + o) = __floats2bfloat162_rn(acc.x, acc.y);
      if (DYf) *reinterpret_cast<float2*>(DYf + o) = acc;
    }
  }
}

// ---------------------------------------------------------------- gate (m-major)
// Y1 [E, G + R*H] with G = L*H gate pre-activations; H1 [E, R*H]:
// H1[e,0,h] = silu(Y1[e, G+h]); H1[e,k,h] = Y1[e, G+k*H+h] * tanh(Y1[e, (l_k-1)*H + h])
template <int L, int MM>
__global__ void gate_fwd_kernel(const __nv_bfloat16* __restrict__ Y1, __nv_bfloat16* __restrict__ H1, int E, int H) {
  using F = Frame<L, MM>;
  constexpr int R = F::R;
  const int e = blockIdx.x;
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= E || h >= H) return;
  const int G = L * H;
  const __nv_bfloat16* y = Y1 + (size_t)e * (G + R * H) + h;
  __nv_bfloat16* o = H1 + (size_t)e * R * H + h;
  float t[L];
#pragma unroll
  for (int l = 1; l <= L; ++l) t[l - 1] = tanhf(bf2f(y[(size_t)(l - 1) * H]));
  o[0] = __float2bfloat16_rn(silu(bf2f(y[G])));
#pragma unroll
  for (int k = 1; k < R; ++k) o[(size_t)k * H] = __float2bfloat16_rn(bf2f(y[G + (size_t)k * H]) * t[F::row_l(k) - 1]);
}

template <int L, int MM>
__global__ void gate_bwd_kernel(const __nv_bfloat16* __restrict__ Y1, const __nv_bfloat16* __restrict__ dH1,
                                __nv_bfloat16* __restrict__ dY1, int E, int H) {
  using F = Frame<L, MM>;
  constexpr int R = F::R;
  const int e = blockIdx.x;
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (e >= E || h >= H) return;
  const int G = L * H;
  const __nv_bfloat16* y = Y1 + (size_t)e * (G + R * H) + h;
  const __nv_bfloat16* dh = dH1 + (size_t)e * R * H + h;
  __nv_bfloat16* dy = dY1 + (size_t)e * (G + R * H) + h;
  float t[L], dg[L];
#pragma unroll
  for (int l = 1; l <= L; ++l) {
    t[l - 1] = tanhf(bf2f(y[(size_t)(l - 1) * H]));
    dg[l - 1] = 0.f;
  }
  dy[G] = __float2bfloat16_rn(bf2f(dh[0]) * dsilu(bf2f(y[G])));
#pragma unroll
  for (int k = 1; k < R; ++k) {
    const int l = F::row_l(k);
    const float d = bf2f(dh[(size_t)k * H]);
    dy[G + (size_t)k * H] = __float2bfloat16_rn(d * t[l - 1]);
    dg[l - 1] += d * bf2f(y[G + (size_t)k * H]);
  }
#pragma unroll
  for (int l = 1; l <= L; ++l) dy[(size_t)(l - 1) * H] = __float2bfloat16_rn(dg[l - 1] * (1.f - t[l - 1] * t[l - 1]));
}

}  // namespace maloq

// ======================================================================= host launchers
namespace maloq {

static const char* last_error() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

// Instantiated frames: lmax 1..6 with mmax in {1, 2, lmax}.
#define MALOQ_FRAME_CASE(L_, M_, ...) \
  if (L == L_ && MM == M_) {          \
    constexpr int FL = L_, FM = M_;   \
    __VA_ARGS__;                      \
    return last_error();              \
  }
#define MALOQ_DISPATCH_FRAME(...)                                                                               \
  MALOQ_FRAME_CASE(1, 1, __VA_ARGS__)                                                                           \
  MALOQ_FRAME_CASE(2, 1, __VA_ARGS__) MALOQ_FRAME_CASE(2, 2, __VA_ARGS__)                                       \
  MALOQ_FRAME_CASE(3, 1, __VA_ARGS__) MALOQ_FRAME_CASE(3, 2, __VA_ARGS__) MALOQ_FRAME_CASE(3, 3, __VA_ARGS__)   \
  MALOQ_FRAME_CASE(4, 1, __VA_ARGS__) MALOQ_FRAME_CASE(4, 2, __VA_ARGS__) MALOQ_FRAME_CASE(4, 4, __VA_ARGS__)   \
  MALOQ_FRAME_CASE(5, 1, __VA_ARGS__) MALOQ_FRAME_CASE(5, 2, __VA_ARGS__) MALOQ_FRAME_CASE(5, 5, __VA_ARGS__)   \
  MALOQ_FRAME_CASE(6, 1, __VA_ARGS__) MALOQ_FRAME_CASE(6, 2, __VA_ARGS__) MALOQ_FRAME_CASE(6, 6, __VA_ARGS__)   \
  return "edge kernels: (lmax, mmax) frame not instantiated (lmax 1..6, mmax in {1, 2, lmax})";

static inline int clampm(int L, int MM) { return MM > L ? L : MM; }

const char* edge_gather_rotate_fwd(int L, int MM, const float* X, const float* XE, const long long* src,
                                   const long long* dst, const float* rot, const __nv_bfloat16* rad,
                                   __nv_bfloat16* A, int E, int C, int Cin, const float* const* peers,
                                   const int* halo_owner, const long long* halo_row, long long n_own,
                                   long long n_x_rows, long long n_halo, cudaStream_t st) {
  MM = clampm(L, MM);
  if (E == 0) return nullptr;
  if (C % 2 != 0) return "gather_rotate: channel count must be even";
  const HaloRef H{peers, halo_owner, halo_row, n_own, peers ? n_own + n_halo : n_x_rows, n_x_rows, nullptr, nullptr};
  MALOQ_DISPATCH_FRAME(({
    constexpr int Q_ = EdgeLanes<(FL + 1) * (FL + 1)>::Q;
    dim3 grid((E + Q_ - 1) / Q_, (Cin / 2 + 63) / 64);
    gather_rotate_fwd_kernel<FL, FM><<<grid, 64 * Q_, 0, st>>>(X, XE, src, dst, rot, rad, A, E, C, Cin, H);
  }))
}

static const char* gather_rotate_bwd_nodes(int L, int MM, const float* X, const float* rot,
                                           const __nv_bfloat16* rad, const __nv_bfloat16* dA,
                                           const long long* dst_ptr, const long long* src_perm,
                                           const long long* src_ptr, float* DX, __nv_bfloat16* DRAD, int N, int E,
                                           int C, int Cin, const HaloRef& H, cudaStream_t st) {
  constexpr int V = 1, Q = 4;
  MALOQ_DISPATCH_FRAME(({
    constexpr int S_ = (FL + 1) * (FL + 1);
    dim3 grid(N, (C / V + 63) / 64);
    gather_rotate_bwd_nodes_kernel<FL, FM, V, Q><<<grid, 64 * Q, (Q - 1) * S_ * 64 * V * sizeof(float), st>>>(
        X, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DRAD, N, C, Cin, E, H);
  }))
}

static const char* gather_rotate_bwd_edges(int L, int MM, const float* XE, const float* rot,
                                           const __nv_bfloat16* rad, const __nv_bfloat16* dA, float* DXE,
                                           __nv_bfloat16* DRAD, int E, int C, int Cin, cudaStream_t st) {
  MALOQ_DISPATCH_FRAME(({
    constexpr int Q_ = EdgeLanes<(FL + 1) * (FL + 1)>::Q;
    dim3 grid((E + Q_ - 1) / Q_, (C / 2 + 63) / 64);
    gather_rotate_bwd_edges_kernel<FL, FM><<<grid, 64 * Q_, 0, st>>>(XE, rot, rad, dA, DXE, DRAD, E, C, Cin);
  }))
}

const char* edge_gather_rotate_bwd(int L, int MM, const float* X, const float* XE, const float* rot,
                                   const __nv_bfloat16* rad, const __nv_bfloat16* dA, const long long* dst_ptr,
                                   const long long* src_perm, const long long* src_ptr, float* DX, float* DXE,
                                   __nv_bfloat16* DRAD, int N, int E, int C, int Cin, const float* const* peers,
                                   const int* halo_owner, const long long* halo_row, long long n_own,
                                   long long n_x_rows, long long n_halo, cudaStream_t st, float* const* recv,
                                   const long long* recv_slot) {
  MM = clampm(L, MM);
  if (C % 2 != 0) return "gather_rotate: channel count must be even";
  if (Cin == 3 * C && (XE == nullptr || DXE == nullptr)) return "gather_rotate_bwd: edge part needs XE and DXE";
  if (recv != nullptr && (peers == nullptr || recv_slot == nullptr)) return "gather_rotate_bwd: recv needs a halo";
  const HaloRef H{peers, halo_owner, halo_row, n_own, peers ? n_own + n_halo : n_x_rows, n_x_rows, recv, recv_slot};
  if (N > 0) {
    const char* err = gather_rotate_bwd_nodes(L, MM, X, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DRAD, N, E, C,
                                              Cin, H, st);
    if (err) return err;
  }
  if (E > 0 && Cin == 3 * C) return gather_rotate_bwd_edges(L, MM, XE, rot, rad, dA, DXE, DRAD, E, C, Cin, st);
  return nullptr;
}

const char* edge_halo_push(const float* G, float* const* recv, const int* halo_owner, const long long* recv_slot,
                           long long n_halo, int SC, cudaStream_t st) {
  if (n_halo == 0) return nullptr;
  if (SC % 4) return "halo push: row size must be a multiple of 4 floats";
  halo_push_kernel<<<(unsigned)n_halo, 128, 0, st>>>(G, recv, halo_owner, recv_slot, n_halo, SC);
  return last_error();
}

const char* edge_halo_fetch(const float* const* peers, const int* halo_owner, const long long* halo_row, float* out,
                            long long n_halo, int SC, cudaStream_t st) {
  if (n_halo == 0) return nullptr;
  if (SC % 4) return "halo fetch: row size must be a multiple of 4 floats";
  halo_fetch_kernel<<<(unsigned)n_halo, 128, 0, st>>>(peers, halo_owner, halo_row, out, n_halo, SC);
  return last_error();
}

const char* edge_node_reduce(const float* DDST, const long long* dst_ptr, const float* DSRC, const long long* src_perm,
                             const long long* src_ptr, float* DX, int N, int SC, long long n_dst_rows,
                             long long n_src_rows, cudaStream_t st) {
  if (N == 0) return nullptr;
  dim3 grid(N, (SC + 255) / 256);
  node_reduce_kernel<<<grid, 256, 0, st>>>(DDST, dst_ptr, DSRC, src_perm, src_ptr, DX, N, SC, n_dst_rows, n_src_rows);
  return last_error();
}

const char* edge_rotate_back_scatter(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot,
                                     const long long* dst_ptr, const float* base, float* out, int N, int C, int Rk,
                                     float scale, cudaStream_t st) {
  MM = clampm(L, MM);
  if (N == 0) return nullptr;
  if (C % 2 == 0 && ldy % 2 == 0 && koff % 2 == 0) {
    dim3 grid(N, (C / 2 + 63) / 64);
    MALOQ_DISPATCH_FRAME(({
      constexpr int S_ = (FL + 1) * (FL + 1), Q_ = EdgeLanes<S_>::Q;
      rotate_back_scatter2_kernel<FL, FM><<<grid, 64 * Q_, (Q_ - 1) * S_ * 64 * sizeof(float2), st>>>(
          Y, ldy, koff, rot, dst_ptr, base, out, N, C, Rk, scale);
    }))
  }
  dim3 grid(N, (C + 127) / 128);
  MALOQ_DISPATCH_FRAME((rotate_back_scatter_kernel<FL, FM><<<grid, 128, 0, st>>>(Y, ldy, koff, rot, dst_ptr, base,
                                                                                  out, N, C, Rk, scale)))
}

const char* edge_rotate_back(int L, int MM, const __nv_bfloat16* Y, int ldy, int koff, const float* rot, float* out,
                             int E, int C, int Rk, cudaStream_t st) {
  MM = clampm(L, MM);
  if (E == 0) return nullptr;
  if (C % 2 == 0 && ldy % 2 == 0 && koff % 2 == 0) {
    MALOQ_DISPATCH_FRAME(({
      constexpr int Q_ = EdgeLanes<(FL + 1) * (FL + 1)>::Q;
      dim3 grid((E + Q_ - 1) / Q_, (C / 2 + 63) / 64);
      rotate_back_edge2_kernel<FL, FM><<<grid, 64 * Q_, 0, st>>>(Y, ldy, koff, rot, out, E, C, Rk);
    }))
  }
  dim3 grid(E, (C + 127) / 128);
  MALOQ_DISPATCH_FRAME((rotate_back_edge_kernel<FL, FM><<<grid, 128, 0, st>>>(Y, ldy, koff, rot, out, E, C, Rk)))
}

const char* edge_rotate_grad(int L, int MM, const float* G, const long long* rows, const float* rot,
                             __nv_bfloat16* DY, float* DYf, int E, int C, int Rk, float scale, cudaStream_t st) {
  MM = clampm(L, MM);
  if (E == 0) return nullptr;
  if (C % 2 == 0) {
    // edge-parallel, two channels per thread; rows (if given) selects each edge's gradient row
    MALOQ_DISPATCH_FRAME(({
      constexpr int Q_ = EdgeLanes<(FL + 1) * (FL + 1)>::Q;
      dim3 grid((E + Q_ - 1) / Q_, (C / 2 + 63) / 64);
      rotate_grad2_kernel<FL, FM, false><<<grid, 64 * Q_, 0, st>>>(G, rows, rot, DY, DYf, E, C, Rk, scale);
    }))
  }
  dim3 grid(E, (C + 127) / 128);
  MALOQ_DISPATCH_FRAME((rotate_grad_kernel<FL, FM><<<grid, 128, 0, st>>>(G, rows, rot, DY, DYf, E, C, Rk, scale)))
}


const char* edge_gate_fwd(int L, int MM, const __nv_bfloat16* Y1, __nv_bfloat16* H1, int E, int H, cudaStream_t st) {
  MM = clampm(L, MM);
  if (E == 0) return nullptr;
  dim3 grid(E, (H + 127) / 128);
  MALOQ_DISPATCH_FRAME((gate_fwd_kernel<FL, FM><<<grid, 128, 0, st>>>(Y1, H1, E, H)))
}

const char* edge_gate_bwd(int L, int MM, const __nv_bfloat16* Y1, const __nv_bfloat16* dH1, __nv_bfloat16* dY1, int E,
                          int H, cudaStream_t st) {
  MM = clampm(L, MM);
  if (E == 0) return nullptr;
  dim3 grid(E, (H + 127) / 128);
  MALOQ_DISPATCH_FRAME((gate_bwd_kernel<FL, FM><<<grid, 128, 0, st>>>(Y1, dH1, dY1, E, H)))
}

}  // namespace maloq
