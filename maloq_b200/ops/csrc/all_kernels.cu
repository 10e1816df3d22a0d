// Unity translation unit of the kernel library: every kernel source is included here so
// that device globals (the error word) have exactly one definition without relocatable
// device code.
#include "runtime.cu"
#include "gemm.cu"
#include "noalloc.cu"
#include "edge.cu"
#include "norm.cu"
#include "comm.cu"
#include "misc.cu"
#include "labels.cu"
#include "graph.cu"
