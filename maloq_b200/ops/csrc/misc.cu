// Per-edge Wigner rotation construction and the fused masked Fock loss.
//
// * edge_rotation: for edge vector v (model frame, polar axis y) with beta = acos(y),
//   alpha = atan2(x, z), writes the rows |m| <= mmax (m-major order) of the block-diagonal
//   D(0, -beta, -alpha) = J X(-beta) J X(-alpha), where X(t) is the rotation about the polar
//   axis (X[a][a] = cos((l-a) t), X[a][2l-a] = sin((l-a) t)) and J the fixed change of axes.
//   One thread per (edge, output row); reference math: helm/common/rotation.py:19-39, 86-99
//   (gamma = 0).  Output ROT [E, R, S] fp32, zero outside the row's degree block.
// * fock_loss_stats / fock_loss_grad: masked squared / absolute error sums of the node and
//   edge label rows (mask = mask_table[pair_type[row]]), reduced per CTA then summed in fixed
//   order; the gradient kernel writes d(loss)/d(output) from the scalar gradients of the
//   statistics, read from device memory (no host round trip between forward and backward).
#include "common.cuh"
#include "misc.h"
#include "edge_inputs.cuh"

namespace maloq {

// rows: row_l[k], row_m[k] (signed m) for the m-major rows; J: concatenated (2l+1)^2 blocks.
struct RotTable {
  int R, S, L;
  int row_l[49];
  int row_m[49];
  int joff[7];
};

__global__ void edge_rotation_kernel(const float* __restrict__ vec, long long ldv, const float* __restrict__ J,
                                     float* __restrict__ ROT, int E, const __grid_constant__ RotTable T) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)E * T.R) return;
  const int k = (int)(idx % T.R);
  const long long e = idx / T.R;
  float x = vec[e * ldv + 0], y = vec[e * ldv + 1], z = vec[e * ldv + 2];
  const float nrm = sqrtf(x * x + y * y + z * z);
  const float inv = nrm > 0.f ? 1.f / nrm : 0.f;
  x *= inv;
  y *= inv;
  z *= inv;
  y = fminf(1.f, fmaxf(-1.f, y));
  const float beta = acosf(y);
  const float alpha = atan2f(x, z);
  const int l = T.row_l[k], d = 2 * l + 1;
  const int i = T.row_m[k] + l;  // row inside the degree block
  const float* Jl = J + T.joff[l];
  float* out = ROT + (e * T.R + k) * T.S;
  for (int j = 0; j < T.S; ++j) out[j] = 0.f;
  // cos/sin of f * angle for f = l - a, a = 0..2l: one sincosf per angle, multiples by the
  // recurrence cos(f t) = 2 cos t cos((f-1) t) - cos((f-2) t) (same for sin), f <= 6
  float cb[13], sb[13], ca[13], sa[13];
  {
    float cbf[7], sbf[7], caf[7], saf[7];
    cbf[0] = caf[0] = 1.f;
    sbf[0] = saf[0] = 0.f;
    sincosf(-beta, &sbf[1], &cbf[1]);
    sincosf(-alpha, &saf[1], &caf[1]);
    for (int f = 2; f <= l; ++f) {
      cbf[f] = 2.f * cbf[1] * cbf[f - 1] - cbf[f - 2];
      sbf[f] = 2.f * cbf[1] * sbf[f - 1] - sbf[f - 2];
      caf[f] = 2.f * caf[1] * caf[f - 1] - caf[f - 2];
      saf[f] = 2.f * caf[1] * saf[f - 1] - saf[f - 2];
    }
    for (int a = 0; a < d; ++a) {
      const int f = l - a;  // cos is even, sin odd in f
      const int af = f < 0 ? -f : f;
      cb[a] = cbf[af];
      ca[a] = caf[af];
      sb[a] = f < 0 ? -sbf[af] : sbf[af];
      sa[a] = f < 0 ? -saf[af] : saf[af];
    }
  }
  // D[i][b] = sum_a J[i][a] * M[a][b],  M = X(-beta) J X(-alpha)
  for (int b = 0; b < d; ++b) {
    float acc = 0.f;
    for (int a = 0; a < d; ++a) {
      const float jia = Jl[i * d + a];
      if (jia == 0.f) continue;
      // M[a][b] = sum_{c in {a, 2l-a}} Xb[a][c] * sum_{q in {b, 2l-b}} J[c][q] Xa[q][b]
      float m = 0.f;
      for (int t = 0; t < 2; ++t) {
        const int c = t == 0 ? a : 2 * l - a;
        if (t == 1 && c == a) break;
        const float xb = (c == a) ? cb[a] : sb[a];
        float inner = 0.f;
        for (int u = 0; u < 2; ++u) {
          const int q = u == 0 ? b : 2 * l - b;
          if (u == 1 && q == b) break;
          // Xa[q][b]: diagonal cos for q == b; for q = 2l-b the row q holds sin((l-q) t) at column b
          const float xa = (q == b) ? ca[q] : sa[q];
          inner += Jl[c * d + q] * xa;
        }
        m += xb * inner;
      }
      acc += jia * m;
    }
    out[l * l + b] = acc;
  }
}

// ---------------------------------------------------------------- loss
// stats per CTA: [sse, sae, cnt] over rows of one output kind (node or edge)
__global__ void fock_loss_stats_kernel(const float* __restrict__ O, const float* __restrict__ Tt,
                                       const long long* __restrict__ pt, const uint8_t* __restrict__ mask, int D,
                                       long long rows, float* __restrict__ part, long long n_pt) {
  float sse = 0.f, sae = 0.f, cnt = 0.f;
  const long long total = rows * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / D;
    const int c = (int)(i - r * D);
    if (MALOQ_IN_BOUNDS(pt[r] >= 0 && pt[r] < n_pt) && mask[pt[r] * D + c]) {
      const float d = O[i] - Tt[i];
      sse += d * d;
      sae += fabsf(d);
      cnt += 1.f;
    }
  }
  __shared__ float red[3][32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sse += __shfl_xor_sync(0xffffffff, sse, o);
    sae += __shfl_xor_sync(0xffffffff, sae, o);
    cnt += __shfl_xor_sync(0xffffffff, cnt, o);
  }
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    red[0][w] = sse;
    red[1][w] = sae;
    red[2][w] = cnt;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float s = 0.f;
    for (int q = 0; q < (int)(blockDim.x / 32); ++q) s += red[threadIdx.x][q];
    part[blockIdx.x * 3 + threadIdx.x] = s;
  }
}

// G[i] = mask * (g_sse * 2 (o - t) + g_sae * sign(o - t))
__global__ void fock_loss_grad_kernel(const float* __restrict__ O, const float* __restrict__ Tt,
                                      const long long* __restrict__ pt, const uint8_t* __restrict__ mask, int D,
                                      long long rows, const float* __restrict__ gstat, float* __restrict__ G,
                                      long long n_pt) {
  const float g_sse = gstat[0], g_sae = gstat[1];
  const long long total = rows * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / D;
    const int c = (int)(i - r * D);
    float g = 0.f;
    if (MALOQ_IN_BOUNDS(pt[r] >= 0 && pt[r] < n_pt) && mask[pt[r] * D + c]) {
      const float d = O[i] - Tt[i];
      g = g_sse * 2.f * d + g_sae * (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f));
    }
    G[i] = g;
  }
}

static const char* misc_err() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

const char* edge_rotation(const float* vec, long long ldv, const float* J, const int* joff, int L, const int* row_l,
                          const int* row_m, int R, float* ROT, int E, cudaStream_t st) {
  if (L > 6 || R > 49) return "edge_rotation: lmax <= 6";
  if (E == 0) return nullptr;
  RotTable T;
  T.R = R;
  T.L = L;
  T.S = (L + 1) * (L + 1);
  for (int k = 0; k < 49; ++k) {
    T.row_l[k] = k < R ? row_l[k] : 0;
    T.row_m[k] = k < R ? row_m[k] : 0;
  }
  for (int l = 0; l < 7; ++l) T.joff[l] = l <= L ? joff[l] : 0;
  const long long n = (long long)E * R;
  edge_rotation_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(vec, ldv, J, ROT, E, T);
  return misc_err();
}

int fock_loss_grid(long long n) { return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 148 * 8)); }

const char* fock_loss_stats(const float* O, const float* Tt, const long long* pt, const uint8_t* mask, int D,
                            long long rows, float* part, int grid, long long n_pt, cudaStream_t st) {
  fock_loss_stats_kernel<<<grid, 256, 0, st>>>(O, Tt, pt, mask, D, rows, part, n_pt);
  return misc_err();
}

const char* fock_loss_grad(const float* O, const float* Tt, const long long* pt, const uint8_t* mask, int D,
                           long long rows, const float* gstat, float* G, long long n_pt, cudaStream_t st) {
  if (rows == 0) return nullptr;
  fock_loss_grad_kernel<<<fock_loss_grid(rows * D), 256, 0, st>>>(O, Tt, pt, mask, D, rows, gstat, G, n_pt);
  return misc_err();
}

const char* edge_inputs(const long long* src_z, const long long* dst_z, const float* D, long long ld_d,
                        const float* src_table, const float* dst_table, long long n_types, const float* offset,
                        float coeff, __nv_bfloat16* OUT, long long E, int C, int NB, cudaStream_t st) {
  if (E == 0) return nullptr;
  const long long total = E * (2LL * C + NB);
  const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 32);
  edge_inputs_kernel<<<grid, 256, 0, st>>>(src_z, dst_z, D, ld_d, src_table, dst_table, n_types, offset, coeff, OUT,
                                           E, C, NB);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace maloq
