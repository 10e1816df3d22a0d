// Python bindings of the maloq_b200 sm_100a kernel library (tensor checks live here; the
// kernel files take raw pointers and a stream).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm.h"
#include "runtime.h"

namespace {

void check(const char* err) { TORCH_CHECK(err == nullptr, "maloq_b200 kernel: ", err ? err : ""); }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// outs[i] = alpha * A[i] @ B[i]^T (+bias) (act); A/B bf16 row-major.
// a_mn=false: A [M,K], B [N,K].  a_mn=true: A [K,M], B [K,N] (weight-gradient form).
// splits > 1: outs[i] is fp32 [splits, M, N] holding partial sums.
void gemm(std::vector<at::Tensor> As, std::vector<at::Tensor> Bs, std::vector<at::Tensor> Cs,
          std::vector<c10::optional<at::Tensor>> biases, bool mn_major, int64_t act, double alpha, int64_t splits,
          int64_t bn) {
  const size_t np = As.size();
  TORCH_CHECK(np >= 1 && np <= 4 && Bs.size() == np && Cs.size() == np, "gemm: 1..4 problems");
  std::vector<maloq::GemmProblem> P(np);
  const bool out_fp32 = Cs[0].scalar_type() == at::kFloat;
  for (size_t i = 0; i < np; ++i) {
    const auto &A = As[i], &B = Bs[i], &C = Cs[i];
    TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors");
    TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
    TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1, "gemm: row-major 2-D A/B");
    TORCH_CHECK((C.scalar_type() == at::kFloat) == out_fp32, "gemm: outputs share a dtype");
    TORCH_CHECK(C.scalar_type() == at::kFloat || C.scalar_type() == at::kBFloat16, "gemm: fp32/bf16 output");
    TORCH_CHECK(C.stride(C.dim() - 1) == 1, "gemm: output rows contiguous");
    auto& g = P[i];
    g.a = A.data_ptr();
    g.lda = A.stride(0);
    g.b = B.data_ptr();
    g.ldb = B.stride(0);
    g.c = C.data_ptr();
    g.M = (int)(mn_major ? A.size(1) : A.size(0));
    g.K = (int)(mn_major ? A.size(0) : A.size(1));
    g.N = (int)(mn_major ? B.size(1) : B.size(0));
    TORCH_CHECK((mn_major ? B.size(0) : B.size(1)) == g.K, "gemm: K mismatch");
    if (splits > 1) {
      TORCH_CHECK(C.dim() == 3 && out_fp32 && C.size(0) == splits && C.size(1) == g.M && C.size(2) == g.N,
                  "gemm: split-K output must be fp32 [splits, M, N]");
      g.ldc = C.stride(1);
      g.split_stride = C.stride(0);
    } else {
      TORCH_CHECK(C.dim() == 2 && C.size(0) == g.M && C.size(1) == g.N, "gemm: output shape");
      g.ldc = C.stride(0);
      g.split_stride = 0;
    }
    g.bias = nullptr;
    if (i < biases.size() && biases[i].has_value()) {
      TORCH_CHECK(biases[i]->scalar_type() == at::kFloat && biases[i]->numel() == g.N, "gemm: fp32 bias [N]");
      g.bias = biases[i]->data_ptr<float>();
    }
  }
  const at::cuda::CUDAGuard guard(As[0].device());
  check(maloq::gemm_launch(P.data(), (int)np, mn_major, mn_major, out_fp32, (int)act, (float)alpha, (int)splits,
                           (int)bn, stream()));
}

void splitk_reduce(at::Tensor part, at::Tensor out, double beta) {
  TORCH_CHECK(part.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat && out.is_contiguous(),
              "splitk_reduce: fp32");
  TORCH_CHECK(part[0].numel() == out.numel(), "splitk_reduce: shape");
  const at::cuda::CUDAGuard guard(part.device());
  check(maloq::gemm_splitk_reduce(part.data_ptr<float>(), out.data_ptr<float>(), out.numel(), (int)part.size(0),
                                  part.stride(0), (float)beta, stream()));
}

int64_t error_status(bool clear) { return maloq::error_status(clear); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &gemm, "grouped tcgen05 bf16 GEMM");
  m.def("splitk_reduce", &splitk_reduce, "sum split-K partials");
  m.def("error_status", &error_status, "read/clear the device error word", py::arg("clear") = true);
}
