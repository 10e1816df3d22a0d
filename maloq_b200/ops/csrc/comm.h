// Host API of comm.cu (NVLink peer-memory collectives).  Plain CUDA types.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace maloq {

// mask = 0: all ranks; otherwise the ranks of the set bits plus this rank (symmetric relation)
const char* peer_barrier(uint32_t* const* pads_dev, int rank, int world, uint32_t epoch, int slot_base,
                         long long spin_limit, cudaStream_t st, unsigned long long mask = 0ull);
// Bucket all-reduce: sum * scale of elements [off, off + n) over ranks, in place.
const char* allreduce_p2p(float* const* bufs_dev, int rank, int world, long long off, long long n, float scale,
                          cudaStream_t st);
const char* allreduce_multimem(float* mc, int rank, int world, long long off, long long n, float scale,
                               cudaStream_t st);

}  // namespace maloq
