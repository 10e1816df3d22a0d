// Intra-node collectives over NVLink peer memory (symmetric-memory buffers).
//
// * peer_barrier: every rank stores `epoch` into slot [rank] of every peer's signal pad
//   (release, system scope) and then waits until its own pad holds `epoch` from every peer
//   (acquire, system scope).  The wait is bounded: on timeout it records ERR_PEER_WAIT and
//   returns, so a missing peer ends the kernel instead of hanging the GPU.
// * allreduce_p2p: rank r owns chunk r of the bucket.  It reads chunk r from every peer
//   buffer (plain loads through peer pointers), sums, scales by `scale`, and stores the result
//   into chunk r of every peer buffer - reduce-scatter and all-gather in one pass, each rank
//   moving 2 (w-1)/w of the bucket over NVLink.
// * allreduce_multimem: the same with NVLink SHARP: one multimem.ld_reduce per vector returns
//   the sum over all ranks (reduced in the switch) and one multimem.st writes it to all ranks.
// Both keep AR_UNROLL vectors per thread in flight.  Usage per bucket, as it becomes ready:
// peer_barrier(epoch) (every rank finished writing the bucket) -> allreduce; one more
// peer_barrier after the step's last bucket, before any rank reads or reuses the buffers.
#include "common.cuh"
#include "comm.h"

namespace maloq {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// mask != 0: only the ranks whose bit is set (and this rank) take part - a barrier among a
// rank's halo neighbours.  The neighbour relation must be symmetric, so every rank that waits
// on another is also signalled by it.
__global__ void peer_barrier_kernel(uint32_t* const* __restrict__ pads, int rank, int world, uint32_t epoch,
                                    int slot_base, long long spin_limit, unsigned long long mask) {
  const int t = threadIdx.x;
  const bool member = t < world && (mask == 0ull || ((mask >> t) & 1ull) || t == rank);
  if (member) {
    __threadfence_system();
    st_release_sys(pads[t] + slot_base + rank, epoch);
  }
  __syncthreads();
  if (member) {
    const uint32_t* mine = pads[rank] + slot_base + t;
    long long i = 0;
    for (; i < spin_limit; ++i) {
      if ((int)(ld_acquire_sys(mine) - epoch) >= 0) break;
      __nanosleep(64);
    }
    if (i == spin_limit) record_error(ERR_PEER_WAIT);
  }
  __syncthreads();
}

constexpr int AR_UNROLL = 4;  // float4 vectors per thread in flight

__global__ void __launch_bounds__(256) allreduce_p2p_kernel(float* const* __restrict__ bufs, int rank, int world,
                                                            long long off, long long n, float scale) {
  const long long chunk = ((n + world - 1) / world + 3) / 4 * 4;
  const long long c0 = off + rank * chunk;
  const long long c1 = off + (rank + 1) * chunk < off + n ? off + (rank + 1) * chunk : off + n;
  const long long nvec = (c1 - c0) / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long v0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; v0 < nvec; v0 += stride * AR_UNROLL) {
    float4 s[AR_UNROLL];
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u) s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      float4 x[AR_UNROLL];
#pragma unroll
      for (int u = 0; u < AR_UNROLL; ++u) {
        const long long v = v0 + u * stride;
        x[u] = v < nvec ? *reinterpret_cast<const float4*>(bufs[p] + c0 + 4 * v) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < AR_UNROLL; ++u) {
        s[u].x += x[u].x;
        s[u].y += x[u].y;
        s[u].z += x[u].z;
        s[u].w += x[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u) {
      s[u].x *= scale;
      s[u].y *= scale;
      s[u].z *= scale;
      s[u].w *= scale;
    }
    for (int p = 0; p < world; ++p)
#pragma unroll
      for (int u = 0; u < AR_UNROLL; ++u) {
        const long long v = v0 + u * stride;
        if (v < nvec) *reinterpret_cast<float4*>(bufs[p] + c0 + 4 * v) = s[u];
      }
  }
  // scalar tail of the chunk
  const long long tail0 = c0 + 4 * nvec;
  for (long long i = tail0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < c1; i += stride) {
    float sum = 0.f;
    for (int p = 0; p < world; ++p) sum += bufs[p][i];
    sum *= scale;
    for (int p = 0; p < world; ++p) bufs[p][i] = sum;
  }
}

__global__ void __launch_bounds__(256) allreduce_multimem_kernel(float* mc, int rank, int world, long long off,
                                                                 long long n, float scale) {
  const long long chunk = ((n + world - 1) / world + 3) / 4 * 4;
  const long long c0 = off + rank * chunk;
  const long long c1 = off + (rank + 1) * chunk < off + n ? off + (rank + 1) * chunk : off + n;
  const long long nvec = (c1 - c0) / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long v0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; v0 < nvec; v0 += stride * AR_UNROLL) {
    float r[AR_UNROLL][4];
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u) {
      const long long v = v0 + u * stride;
      if (v < nvec) {
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(r[u][0]), "=f"(r[u][1]), "=f"(r[u][2]), "=f"(r[u][3])
                     : "l"(mc + c0 + 4 * v)
                     : "memory");
      }
    }
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u) {
      const long long v = v0 + u * stride;
      if (v < nvec)
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc + c0 + 4 * v),
                     "f"(r[u][0] * scale), "f"(r[u][1] * scale), "f"(r[u][2] * scale), "f"(r[u][3] * scale)
                     : "memory");
    }
  }
  const long long tail0 = c0 + 4 * nvec;
  for (long long i = tail0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < c1; i += stride) {
    float a;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(a) : "l"(mc + i) : "memory");
    a *= scale;
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc + i), "f"(a) : "memory");
  }
}

static const char* comm_err() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

const char* peer_barrier(uint32_t* const* pads_dev, int rank, int world, uint32_t epoch, int slot_base,
                         long long spin_limit, cudaStream_t st, unsigned long long mask) {
  if (world > 1024) return "peer_barrier: world too large";
  if (mask != 0ull && world > 64) return "peer_barrier: a member mask needs world <= 64";
  peer_barrier_kernel<<<1, world < 32 ? 32 : world, 0, st>>>(pads_dev, rank, world, epoch, slot_base, spin_limit,
                                                                mask);
  return comm_err();
}

static int ar_blocks(long long n, int world) {
  const long long per = (n + world - 1) / world / 4 + 1;
  long long blocks = (per + 256 * AR_UNROLL - 1) / (256 * AR_UNROLL);
  if (blocks > 148 * 2) blocks = 148 * 2;
  return blocks < 1 ? 1 : (int)blocks;
}

const char* allreduce_p2p(float* const* bufs_dev, int rank, int world, long long off, long long n, float scale,
                          cudaStream_t st) {
  if (n == 0) return nullptr;
  allreduce_p2p_kernel<<<ar_blocks(n, world), 256, 0, st>>>(bufs_dev, rank, world, off, n, scale);
  return comm_err();
}

const char* allreduce_multimem(float* mc, int rank, int world, long long off, long long n, float scale,
                               cudaStream_t st) {
  if (n == 0) return nullptr;
  allreduce_multimem_kernel<<<ar_blocks(n, world), 256, 0, st>>>(mc, rank, world, off, n, scale);
  return comm_err();
}

}  // namespace maloq
