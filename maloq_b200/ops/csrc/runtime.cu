// Library-wide device state: the error word written by bounded waits and bounds checks.
#include "common.cuh"
#include "runtime.h"

namespace maloq {

int error_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_maloq_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    int z = 0;
    if (cudaMemcpyToSymbol(g_maloq_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

bool bounds_checked() { return MALOQ_BOUNDS_CHECKED != 0; }

}  // namespace maloq
