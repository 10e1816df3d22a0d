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
// * colsum: column sums of a row-strided [M, N] fp32 or bf16 matrix into fp32 [N] (bias
//   gradients, per-CTA partial sums of the norm kernels) in a fixed order, so that the result
//   does not depend on scheduling.  Stage 1: a 32 x 8 CTA covers 32 columns of one row chunk;
//   each thread sums every 8th row of the chunk with four independent accumulators, the 8
//   partials are added in thread order through shared memory into part[chunk, N].  Stage 2
//   is the same kernel over part with a single chunk.  One stage when the matrix is short.
//   colsum_segments: one CTA row per row segment (per-degree sums of split-K partials).
// * weight_pack: the bf16 GEMM operand copies of fp32 master weights (plain, transposed, and
//   the SO(2) pair matrix [[W_r, -W_i], [W_i, W_r]] of W = [W_r; W_i] and its transpose), and
//   the fp32 gradient of W from the gradient of its pair matrix, for up to kPackJobs tensors in
//   one launch: the job table is a kernel parameter, each thread writes one output element
//   (coalesced stores) and finds its job by a binary search over the jobs' first elements.
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

__device__ __forceinline__ float colsum_load(const float* p) { return *p; }
__device__ __forceinline__ float colsum_load(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// CTA: 32 columns from blockIdx.x, rows [r0, r1); writes the 32 sums to out[n]
template <class T>
__device__ __forceinline__ void colsum_block(const T* __restrict__ X, long long r0, long long r1, int N, long long ld,
                                             float* __restrict__ out) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int n = blockIdx.x * 32 + tx;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (n < N) {
    const T* p = X + n;
    long long r = r0 + ty;
    for (; r + 24 < r1; r += 32) {
      s0 += colsum_load(p + r * ld);
      s1 += colsum_load(p + (r + 8) * ld);
      s2 += colsum_load(p + (r + 16) * ld);
      s3 += colsum_load(p + (r + 24) * ld);
    }
    for (; r < r1; r += 8) s0 += colsum_load(p + r * ld);
  }
  red[ty][tx] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (ty == 0 && n < N) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k][tx];
    out[n] = t;
  }
}

// blockIdx.y: row chunk [y * chunk, (y + 1) * chunk) -> out row y
template <class T>
__global__ void __launch_bounds__(256) colsum_kernel(const T* __restrict__ X, long long M, int N, long long ld,
                                                     long long chunk, float* __restrict__ out) {
  const long long r0 = blockIdx.y * chunk;
  colsum_block(X, r0, r0 + chunk < M ? r0 + chunk : M, N, ld, out + blockIdx.y * (long long)N);
}

struct SegTable {
  long long ptr[kColsumSegs + 1];
};

// blockIdx.y: row segment [ptr[y], ptr[y + 1]) -> out row y
__global__ void __launch_bounds__(256) colsum_seg_kernel(const float* __restrict__ X, int N, long long ld,
                                                         const __grid_constant__ SegTable T, float* __restrict__ out) {
  colsum_block(X, T.ptr[blockIdx.y], T.ptr[blockIdx.y + 1], N, ld, out + blockIdx.y * (long long)N);
}

struct PackTable {
  int n;
  long long start[kPackJobs + 1];  // first output element of each job; start[n] = total
  const float* src[kPackJobs];
  void* dst[kPackJobs];
  int batch[kPackJobs], rows[kPackJobs], cols[kPackJobs], kind[kPackJobs];  // shape of src
};

__global__ void __launch_bounds__(256) weight_pack_kernel(const __grid_constant__ PackTable T) {
  const long long total = T.start[T.n];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int lo = 0, hi = T.n - 1;  // last job with start <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (T.start[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int j = lo;
    const long long t = i - T.start[j];
    const int rows = T.rows[j], cols = T.cols[j], kind = T.kind[j];
    const float* S = T.src[j];
    float v;
    if (kind == kPackCast) {
      v = S[t];
    } else if (kind == kPackTranspose) {  // dst [batch, cols, rows]
      const long long mat = (long long)rows * cols, b = t / mat, u = t % mat;
      const int x = (int)(u / rows), y = (int)(u % rows);
      v = S[b * mat + (long long)y * cols + x];
    } else if (kind == kPackPairGrad) {  // src dP [2h, 2k] -> dst fp32 [2h, k]
      const int h = rows / 2, k = cols / 2;
      const int R = (int)(t / k), c = (int)(t % k), r = R % h;
      v = R < h ? S[(long long)r * cols + c] + S[(long long)(h + r) * cols + k + c]
                : S[(long long)(h + r) * cols + c] - S[(long long)r * cols + k + c];
      static_cast<float*>(T.dst[j])[t] = v;
      continue;
    } else {  // pair matrix [2h, 2k] of src [2h, k] (kPackPair), or its transpose [2k, 2h]
      const int h = rows / 2, k = cols;
      int R, C;
      if (kind == kPackPair) {
        R = (int)(t / (2 * k));
        C = (int)(t % (2 * k));
      } else {
        C = (int)(t / (2 * h));
        R = (int)(t % (2 * h));
      }
      const int a = R / h, r = R % h, q = C / k, c = C % k;
      // (a, q) = (0, 0): W_r   (0, 1): -W_i   (1, 0): W_i   (1, 1): W_r
      const float w = S[(long long)((a ^ q) ? h + r : r) * k + c];
      v = (a == 0 && q == 1) ? -w : w;
    }
    static_cast<__nv_bfloat16*>(T.dst[j])[t] = __float2bfloat16(v);
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

int colsum_chunks(long long M, int N) {
  if (M <= 4096) return 1;
  const long long cols = (N + 31) / 32;
  const long long want = (148 * 4 + cols - 1) / cols;  // about four CTAs per SM in stage 1
  const long long most = (M + 255) / 256;              // at least 256 rows (32 per thread) a chunk
  return (int)std::max<long long>(1, std::min<long long>(std::min(want, most), 1024));
}

const char* colsum(const void* X, bool bf16, long long M, int N, long long ld, float* part, int P, float* out,
                   cudaStream_t st) {
  if (N <= 0) return nullptr;
  const dim3 blk(32, 8);
  if (P <= 1 || M == 0) {
    const long long chunk = M > 0 ? M : 1;
    if (bf16)
      colsum_kernel<__nv_bfloat16><<<dim3((N + 31) / 32, 1), blk, 0, st>>>(static_cast<const __nv_bfloat16*>(X), M, N, ld, chunk,
                                                            out);
    else
      colsum_kernel<float><<<dim3((N + 31) / 32, 1), blk, 0, st>>>(static_cast<const float*>(X), M, N, ld, chunk, out);
    return misc_err();
  }
  const long long chunk = (M + P - 1) / P;
  // chunks that hold rows (<= P): stage 2 reads only the rows of part that stage 1 wrote
  const int used = (int)((M + chunk - 1) / chunk);
  if (bf16)
    colsum_kernel<__nv_bfloat16><<<dim3((N + 31) / 32, used), blk, 0, st>>>(static_cast<const __nv_bfloat16*>(X), M, N, ld, chunk,
                                                             part);
  else
    colsum_kernel<float><<<dim3((N + 31) / 32, used), blk, 0, st>>>(static_cast<const float*>(X), M, N, ld, chunk, part);
  colsum_kernel<float><<<dim3((N + 31) / 32, 1), blk, 0, st>>>(static_cast<const float*>(part), (long long)used, N,
                                                        (long long)N, (long long)used, out);
  return misc_err();
}

const char* colsum_segments(const float* X, int N, long long ld, const long long* seg, int nseg, float* out,
                            cudaStream_t st) {
  if (nseg < 1 || nseg > kColsumSegs) return "colsum_segments: 1 to kColsumSegs segments";
  if (N <= 0) return nullptr;
  SegTable T;
  for (int s = 0; s <= nseg; ++s) {
    T.ptr[s] = seg[s];
    if (s > 0 && seg[s] < seg[s - 1]) return "colsum_segments: decreasing row offsets";
  }
  colsum_seg_kernel<<<dim3((N + 31) / 32, nseg), dim3(32, 8), 0, st>>>(X, N, ld, T, out);
  return misc_err();
}

const char* weight_pack(int n, const float* const* src, void* const* dst, const int* batch, const int* rows,
                        const int* cols, const int* kind, cudaStream_t st) {
  for (int j0 = 0; j0 < n; j0 += kPackJobs) {
    PackTable T;
    T.n = std::min(kPackJobs, n - j0);
    long long at = 0;
    for (int j = 0; j < T.n; ++j) {
      const int g = j0 + j, kd = kind[g];
      if (kd < kPackCast || kd > kPackPairGrad) return "weight_pack: unknown job kind";
      if ((kd == kPackPair || kd == kPackPairT || kd == kPackPairGrad) && (rows[g] % 2 || batch[g] != 1))
        return "weight_pack: a pair job needs one matrix with an even row count";
      if (kd == kPackPairGrad && cols[g] % 2) return "weight_pack: a pair gradient needs an even column count";
      T.start[j] = at;
      T.src[j] = src[g];
      T.dst[j] = dst[g];
      T.batch[j] = batch[g];
      T.rows[j] = rows[g];
      T.cols[j] = cols[g];
      T.kind[j] = kd;
      const long long m = (long long)batch[g] * rows[g] * cols[g];
      at += (kd == kPackPair || kd == kPackPairT) ? 2 * m : (kd == kPackPairGrad ? m / 2 : m);
    }
    T.start[T.n] = at;
    if (at == 0) continue;
    const int grid = (int)std::min<long long>((at + 255) / 256, 148 * 8);
    weight_pack_kernel<<<grid, 256, 0, st>>>(T);
    const char* e = misc_err();
    if (e) return e;
  }
  return nullptr;
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
