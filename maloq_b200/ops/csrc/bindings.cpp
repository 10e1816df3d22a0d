// Python bindings of the maloq_b200 sm_100a kernel library (tensor checks live here; the
// kernel files take raw pointers and a stream).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "comm.h"
#include "edge.h"
#include "gemm.h"
#include "graph.h"
#include "labels.h"
#include "misc.h"
#include "norm.h"
#include "runtime.h"

namespace {

void check(const char* err) { TORCH_CHECK(err == nullptr, "maloq_b200 kernel: ", err ? err : ""); }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// outs[i] = alpha * A[i] @ B[i]^T (+bias) (act); A/B bf16 row-major.
// a_mn=false: A [M,K], B [N,K].  a_mn=true: A [K,M], B [K,N] (weight-gradient form).
// splits > 1: outs[i] is fp32 [splits, M, N] holding partial sums.
// resids (optional, fp32 output only): Rs[i] [M,N] (row stride free) added in the epilogue.
void gemm(std::vector<at::Tensor> As, std::vector<at::Tensor> Bs, std::vector<at::Tensor> Cs,
          std::vector<c10::optional<at::Tensor>> biases, bool mn_major, int64_t act, double alpha, int64_t splits,
          int64_t bn, std::vector<c10::optional<at::Tensor>> resids) {
  const size_t np = As.size();
  TORCH_CHECK(np >= 1 && np <= 8 && Bs.size() == np && Cs.size() == np, "gemm: 1..8 problems");
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
    if (splits > 1 || C.dim() == 3) {
      TORCH_CHECK(C.dim() == 3 && out_fp32 && C.size(0) == splits && C.size(1) == g.M && C.size(2) == g.N,
                  "gemm: split-K output must be fp32 [splits, M, N]");
      g.ldc = C.stride(1);
      g.split_stride = C.stride(0);
    } else {
      TORCH_CHECK(C.dim() == 2 && C.size(0) == g.M && C.size(1) == g.N, "gemm: output shape");
      g.ldc = C.stride(0);
      g.split_stride = 0;
    }
    if (i < resids.size() && resids[i].has_value()) {
      const auto& R = *resids[i];
      TORCH_CHECK(R.scalar_type() == at::kFloat && out_fp32 && R.dim() == 2 && R.size(0) == g.M &&
                      R.size(1) == g.N && R.stride(1) == 1,
                  "gemm: residual must be fp32 [M, N] with contiguous rows (fp32 output)");
      g.resid = R.data_ptr<float>();
      g.ldr = R.stride(0);
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


template <class T>
T* ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr<T>() : nullptr;
}

void chk(const at::Tensor& t, at::ScalarType dt, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == dt, what,
              ": expected a contiguous CUDA tensor of ", dt);
}

__nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
const long long* ll(const at::Tensor& t) { return reinterpret_cast<const long long*>(t.data_ptr<int64_t>()); }
const long long* ll(const c10::optional<at::Tensor>& t) { return t.has_value() ? ll(*t) : nullptr; }

// A [E, R*Cin] = rad * rot . [X[src] | X[dst] | XE]; rad bf16 [E, NS*Cin]
void gather_rotate_fwd(int64_t L, int64_t MM, at::Tensor X, c10::optional<at::Tensor> XE, at::Tensor src,
                       at::Tensor dst, at::Tensor rot, c10::optional<at::Tensor> rad, at::Tensor A, int64_t Cin,
                       int64_t peers, c10::optional<at::Tensor> halo_owner, c10::optional<at::Tensor> halo_row,
                       int64_t n_own) {
  chk(X, at::kFloat, "X");
  chk(rot, at::kFloat, "rot");
  chk(A, at::kBFloat16, "A");
  chk(src, at::kLong, "src");
  chk(dst, at::kLong, "dst");
  if (XE.has_value()) chk(*XE, at::kFloat, "XE");
  if (rad.has_value()) chk(*rad, at::kBFloat16, "rad");
  TORCH_CHECK(A.numel() == src.numel() * rot.size(1) * Cin, "gather_rotate_fwd: A must be [E, R*Cin]");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::edge_gather_rotate_fwd((int)L, (int)MM, X.data_ptr<float>(), ptr<float>(XE), ll(src), ll(dst),
                                      rot.data_ptr<float>(), rad.has_value() ? bf(*rad) : nullptr, bf(A),
                                      (int)src.size(0), (int)X.size(2), (int)Cin,
                                      reinterpret_cast<const float* const*>(peers),
                                      halo_owner.has_value() ? halo_owner->data_ptr<int>() : nullptr, ll(halo_row),
                                      n_own, X.size(0), halo_owner.has_value() ? halo_owner->numel() : 0, stream()));
}

// Backward of gather_rotate: node gradients DX [N, S, C] (dst CSR + src CSR walks, no per-edge
// rows), DXE (edge embedding part), DRAD (bf16)
void gather_rotate_bwd(int64_t L, int64_t MM, at::Tensor X, c10::optional<at::Tensor> XE, at::Tensor rot,
                       c10::optional<at::Tensor> rad, at::Tensor dA, at::Tensor dst_ptr, at::Tensor src_perm,
                       at::Tensor src_ptr, at::Tensor DX, c10::optional<at::Tensor> DXE,
                       c10::optional<at::Tensor> DRAD, int64_t Cin, int64_t peers,
                       c10::optional<at::Tensor> halo_owner, c10::optional<at::Tensor> halo_row, int64_t n_own,
                       int64_t recv, c10::optional<at::Tensor> recv_slot) {
  chk(X, at::kFloat, "X");
  chk(rot, at::kFloat, "rot");
  chk(dA, at::kBFloat16, "dA");
  chk(DX, at::kFloat, "DX");
  chk(dst_ptr, at::kLong, "dst_ptr");
  chk(src_perm, at::kLong, "src_perm");
  chk(src_ptr, at::kLong, "src_ptr");
  if (rad.has_value()) chk(*rad, at::kBFloat16, "rad");
  if (DRAD.has_value()) chk(*DRAD, at::kBFloat16, "DRAD");
  if (XE.has_value()) chk(*XE, at::kFloat, "XE");
  if (DXE.has_value()) chk(*DXE, at::kFloat, "DXE");
  const int N = (int)DX.size(0);
  TORCH_CHECK(dst_ptr.numel() == N + 1 && src_ptr.numel() == N + 1, "gather_rotate_bwd: CSR offsets need N+1 rows");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::edge_gather_rotate_bwd((int)L, (int)MM, X.data_ptr<float>(), ptr<float>(XE), rot.data_ptr<float>(),
                                      rad.has_value() ? bf(*rad) : nullptr, bf(dA), ll(dst_ptr), ll(src_perm),
                                      ll(src_ptr), DX.data_ptr<float>(), ptr<float>(DXE),
                                      DRAD.has_value() ? bf(*DRAD) : nullptr, N, (int)rot.size(0), (int)X.size(2),
                                      (int)Cin, reinterpret_cast<const float* const*>(peers),
                                      halo_owner.has_value() ? halo_owner->data_ptr<int>() : nullptr, ll(halo_row),
                                      n_own, X.size(0), halo_owner.has_value() ? halo_owner->numel() : 0, stream(),
                                      reinterpret_cast<float* const*>(recv), ll(recv_slot)));
}

// DX[n] = sum over dst-CSR of DDST + sum over src-CSR of DSRC (either may be absent)
// OUT[h] = row halo_row[h] of rank halo_owner[h]'s staging slot (peers = device table of slot bases)
void halo_fetch(int64_t peers, at::Tensor halo_owner, at::Tensor halo_row, at::Tensor OUT) {
  chk(OUT, at::kFloat, "halo_fetch out");
  chk(halo_owner, at::kInt, "halo_owner");
  chk(halo_row, at::kLong, "halo_row");
  TORCH_CHECK(OUT.size(0) == halo_owner.numel() && halo_row.numel() == halo_owner.numel(), "halo_fetch: rows");
  const at::cuda::CUDAGuard guard(OUT.device());
  check(maloq::edge_halo_fetch(reinterpret_cast<const float* const*>(peers), halo_owner.data_ptr<int>(), ll(halo_row),
                               OUT.data_ptr<float>(), OUT.size(0), (int)(OUT.numel() / std::max<int64_t>(1, OUT.size(0))),
                               stream()));
}

void halo_push(at::Tensor G, int64_t recv, at::Tensor halo_owner, at::Tensor recv_slot) {
  chk(G, at::kFloat, "G");
  const int SC = (int)(G.numel() / std::max<int64_t>(1, G.size(0)));
  const at::cuda::CUDAGuard guard(G.device());
  check(maloq::edge_halo_push(G.data_ptr<float>(), reinterpret_cast<float* const*>(recv), halo_owner.data_ptr<int>(),
                              ll(recv_slot), G.size(0), SC, stream()));
}

void node_reduce(c10::optional<at::Tensor> DDST, at::Tensor dst_ptr, c10::optional<at::Tensor> DSRC,
                 c10::optional<at::Tensor> src_perm, c10::optional<at::Tensor> src_ptr, at::Tensor DX) {
  chk(DX, at::kFloat, "DX");
  const int N = (int)DX.size(0);
  const int SC = (int)(DX.numel() / std::max<int64_t>(1, N));
  const at::cuda::CUDAGuard guard(DX.device());
  check(maloq::edge_node_reduce(ptr<float>(DDST), ll(dst_ptr), ptr<float>(DSRC), ll(src_perm), ll(src_ptr),
                                DX.data_ptr<float>(), N, SC, DDST.has_value() ? DDST->size(0) : 0,
                                DSRC.has_value() ? DSRC->size(0) : 0, stream()));
}

void rotate_back_scatter(int64_t L, int64_t MM, at::Tensor Y, int64_t koff, int64_t Rk, at::Tensor rot,
                         at::Tensor dst_ptr, c10::optional<at::Tensor> base, at::Tensor out, double scale) {
  chk(Y, at::kBFloat16, "Y");
  chk(out, at::kFloat, "out");
  if (base.has_value()) chk(*base, at::kFloat, "base");
  const at::cuda::CUDAGuard guard(Y.device());
  check(maloq::edge_rotate_back_scatter((int)L, (int)MM, bf(Y), (int)Y.size(1), (int)koff, rot.data_ptr<float>(),
                                        ll(dst_ptr), ptr<float>(base), out.data_ptr<float>(), (int)out.size(0),
                                        (int)out.size(2), (int)Rk, (float)scale, stream()));
}

void rotate_back_edge(int64_t L, int64_t MM, at::Tensor Y, int64_t koff, int64_t Rk, at::Tensor rot, at::Tensor out) {
  chk(Y, at::kBFloat16, "Y");
  chk(out, at::kFloat, "out");
  const at::cuda::CUDAGuard guard(Y.device());
  check(maloq::edge_rotate_back((int)L, (int)MM, bf(Y), (int)Y.size(1), (int)koff, rot.data_ptr<float>(),
                                out.data_ptr<float>(), (int)out.size(0), (int)out.size(2), (int)Rk, stream()));
}

void rotate_grad(int64_t L, int64_t MM, at::Tensor G, c10::optional<at::Tensor> rows, at::Tensor rot,
                 c10::optional<at::Tensor> DY, c10::optional<at::Tensor> DYf, int64_t Rk, double scale) {
  chk(G, at::kFloat, "G");
  const at::cuda::CUDAGuard guard(G.device());
  check(maloq::edge_rotate_grad((int)L, (int)MM, G.data_ptr<float>(), ll(rows), rot.data_ptr<float>(),
                                DY.has_value() ? bf(*DY) : nullptr, ptr<float>(DYf), (int)rot.size(0),
                                (int)G.size(2), (int)Rk, (float)scale, stream()));
}

void gate_fwd(int64_t L, int64_t MM, at::Tensor Y1, at::Tensor H1, int64_t H) {
  chk(Y1, at::kBFloat16, "Y1");
  chk(H1, at::kBFloat16, "H1");
  const at::cuda::CUDAGuard guard(Y1.device());
  check(maloq::edge_gate_fwd((int)L, (int)MM, bf(Y1), bf(H1), (int)Y1.size(0), (int)H, stream()));
}

void gate_bwd(int64_t L, int64_t MM, at::Tensor Y1, at::Tensor dH1, at::Tensor dY1, int64_t H) {
  chk(Y1, at::kBFloat16, "Y1");
  chk(dH1, at::kBFloat16, "dH1");
  chk(dY1, at::kBFloat16, "dY1");
  const at::cuda::CUDAGuard guard(Y1.device());
  check(maloq::edge_gate_bwd((int)L, (int)MM, bf(Y1), bf(dH1), bf(dY1), (int)Y1.size(0), (int)H, stream()));
}


// OUT fp32 or bf16 (the dtype of the tensor passed)
void rms_norm_fwd(int64_t L, at::Tensor X, c10::optional<at::Tensor> RES, at::Tensor aw, at::Tensor ab,
                  at::Tensor OUT, c10::optional<at::Tensor> SUM, double eps) {
  chk(X, at::kFloat, "X");
  const bool ob = OUT.scalar_type() == at::kBFloat16;
  chk(OUT, ob ? at::kBFloat16 : at::kFloat, "OUT");
  chk(aw, at::kFloat, "affine_weight");
  chk(ab, at::kFloat, "affine_bias");
  if (RES.has_value()) chk(*RES, at::kFloat, "RES");
  if (SUM.has_value()) chk(*SUM, at::kFloat, "SUM");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::rms_norm_fwd((int)L, X.data_ptr<float>(), ptr<float>(RES), aw.data_ptr<float>(), ab.data_ptr<float>(),
                            OUT.data_ptr(), ob, ptr<float>(SUM), (int)X.size(0), (int)X.size(2), (float)eps,
                            stream()));
}

// G fp32 or bf16
void rms_norm_bwd(int64_t L, at::Tensor Sx, at::Tensor G, c10::optional<at::Tensor> GS, at::Tensor aw, at::Tensor DX,
                  at::Tensor PART, double eps) {
  chk(Sx, at::kFloat, "S");
  const bool gb = G.scalar_type() == at::kBFloat16;
  chk(G, gb ? at::kBFloat16 : at::kFloat, "G");
  chk(DX, at::kFloat, "DX");
  chk(PART, at::kFloat, "PART");
  if (GS.has_value()) chk(*GS, at::kFloat, "GS");
  const at::cuda::CUDAGuard guard(Sx.device());
  check(maloq::rms_norm_bwd((int)L, Sx.data_ptr<float>(), G.data_ptr(), gb, ptr<float>(GS), aw.data_ptr<float>(),
                            DX.data_ptr<float>(), PART.data_ptr<float>(), (int)Sx.size(0), (int)Sx.size(2), (float)eps,
                            (int)PART.size(0), stream()));
}

int64_t norm_grid(int64_t rows) { return maloq::norm_grid(rows); }

void ln_silu_fwd(at::Tensor X, at::Tensor w, at::Tensor b, at::Tensor OUT, double eps) {
  chk(X, at::kFloat, "X");
  chk(OUT, at::kBFloat16, "OUT");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::ln_silu_fwd(X.data_ptr<float>(), w.data_ptr<float>(), b.data_ptr<float>(), bf(OUT), (int)X.size(0),
                           (int)X.size(1), (float)eps, stream()));
}

void ln_silu_bwd(at::Tensor X, at::Tensor w, at::Tensor b, at::Tensor G, at::Tensor DX, at::Tensor PART, double eps) {
  chk(X, at::kFloat, "X");
  chk(G, at::kBFloat16, "G");
  chk(DX, at::kFloat, "DX");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::ln_silu_bwd(X.data_ptr<float>(), w.data_ptr<float>(), b.data_ptr<float>(), bf(G), DX.data_ptr<float>(),
                           PART.data_ptr<float>(), (int)X.size(0), (int)X.size(1), (float)eps,
                           (int)(PART.size(0) / 8), stream()));
}

// X / OUT (and DO / DX) share a dtype, fp32 or bf16; gates fp32
void gate_l_fwd(int64_t L, at::Tensor X, at::Tensor Gt, at::Tensor OUT, bool silu_gates) {
  const bool b16 = X.scalar_type() == at::kBFloat16;
  chk(X, b16 ? at::kBFloat16 : at::kFloat, "X");
  chk(Gt, at::kFloat, "gates");
  chk(OUT, b16 ? at::kBFloat16 : at::kFloat, "OUT");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::gate_l_fwd((int)L, X.data_ptr(), Gt.data_ptr<float>(), OUT.data_ptr(), b16, (int)X.size(0),
                          (int)X.size(2), stream(), silu_gates));
}

void gate_l_bwd(int64_t L, at::Tensor X, at::Tensor Gt, at::Tensor DO, at::Tensor DX, at::Tensor DG, bool silu_gates) {
  const bool b16 = X.scalar_type() == at::kBFloat16;
  chk(X, b16 ? at::kBFloat16 : at::kFloat, "X");
  chk(DO, b16 ? at::kBFloat16 : at::kFloat, "DO");
  chk(DX, b16 ? at::kBFloat16 : at::kFloat, "DX");
  chk(Gt, at::kFloat, "gates");
  chk(DG, at::kFloat, "DG");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::gate_l_bwd((int)L, X.data_ptr(), Gt.data_ptr<float>(), DO.data_ptr(), DX.data_ptr(),
                          DG.data_ptr<float>(), b16, (int)X.size(0), (int)X.size(2), stream(), silu_gates));
}

// Fock-head gate: X [B, S, C] fp32, SV [B, (L+1) C] fp32, A [B, S, C] bf16 (act 0 sigmoid, 1 tanh)
static void head_gate_shapes(int64_t L, const at::Tensor& X, const at::Tensor& SV) {
  const int64_t S = (L + 1) * (L + 1);
  TORCH_CHECK(X.dim() == 3 && X.size(1) == S, "head_gate: X must be [B, (L+1)^2, C]");
  TORCH_CHECK(SV.dim() == 2 && SV.size(0) == X.size(0) && SV.size(1) == (L + 1) * X.size(2),
              "head_gate: SV must be [B, (L+1) C]");
}

void head_gate_fwd(int64_t L, at::Tensor X, at::Tensor SV, at::Tensor A, int64_t act, double scale, bool absg) {
  chk(X, at::kFloat, "X");
  chk(SV, at::kFloat, "SV");
  chk(A, at::kBFloat16, "A");
  head_gate_shapes(L, X, SV);
  TORCH_CHECK(A.sizes() == X.sizes(), "head_gate_fwd: A must have X's shape");
  TORCH_CHECK(act == 0 || act == 1, "head_gate: act must be 0 (sigmoid) or 1 (tanh)");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::head_gate_fwd((int)L, X.data_ptr<float>(), SV.data_ptr<float>(), bf(A), (int)act, (float)scale, absg,
                             (int)X.size(0), (int)X.size(2), stream()));
}

void head_gate_bwd(int64_t L, at::Tensor X, at::Tensor SV, at::Tensor DA, at::Tensor DX, at::Tensor DSV, int64_t act,
                   double scale, bool absg) {
  chk(X, at::kFloat, "X");
  chk(SV, at::kFloat, "SV");
  chk(DA, at::kFloat, "DA");
  chk(DX, at::kFloat, "DX");
  chk(DSV, at::kFloat, "DSV");
  head_gate_shapes(L, X, SV);
  TORCH_CHECK(DA.sizes() == X.sizes() && DX.sizes() == X.sizes() && DSV.sizes() == SV.sizes(),
              "head_gate_bwd: DA / DX must have X's shape, DSV SV's");
  TORCH_CHECK(act == 0 || act == 1, "head_gate: act must be 0 (sigmoid) or 1 (tanh)");
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::head_gate_bwd((int)L, X.data_ptr<float>(), SV.data_ptr<float>(), DA.data_ptr<float>(),
                             DX.data_ptr<float>(), DSV.data_ptr<float>(), (int)act, (float)scale, absg, (int)X.size(0),
                             (int)X.size(2), stream()));
}


// ---- NVLink peer-memory collectives (pointers come from torch symmetric memory handles)
void peer_barrier(int64_t pads_dev, int64_t rank, int64_t world, int64_t epoch, int64_t slot_base, int64_t spin_limit) {
  check(maloq::peer_barrier(reinterpret_cast<uint32_t* const*>(pads_dev), (int)rank, (int)world, (uint32_t)epoch,
                            (int)slot_base, spin_limit, stream()));
}

// barrier among this rank's halo neighbours (bit t of mask set for neighbour t; world <= 64)
void peer_barrier_mask(int64_t pads_dev, int64_t rank, int64_t world, int64_t epoch, int64_t slot_base,
                       int64_t spin_limit, int64_t mask) {
  check(maloq::peer_barrier(reinterpret_cast<uint32_t* const*>(pads_dev), (int)rank, (int)world, (uint32_t)epoch,
                            (int)slot_base, spin_limit, stream(), (unsigned long long)mask));
}

void allreduce_p2p(int64_t bufs_dev, int64_t rank, int64_t world, int64_t off, int64_t n, double scale) {
  check(maloq::allreduce_p2p(reinterpret_cast<float* const*>(bufs_dev), (int)rank, (int)world, off, n, (float)scale,
                             stream()));
}

void allreduce_multimem(int64_t mc, int64_t rank, int64_t world, int64_t off, int64_t n, double scale) {
  check(maloq::allreduce_multimem(reinterpret_cast<float*>(mc), (int)rank, (int)world, off, n, (float)scale, stream()));
}


void edge_rotation(at::Tensor vec, at::Tensor J, std::vector<int64_t> joff, int64_t L, std::vector<int64_t> row_l,
                   std::vector<int64_t> row_m, at::Tensor ROT) {
  TORCH_CHECK(vec.is_cuda() && vec.scalar_type() == at::kFloat && vec.stride(1) == 1, "edge_rotation: fp32 vec [E,3]");
  chk(J, at::kFloat, "J");
  chk(ROT, at::kFloat, "ROT");
  std::vector<int> jo(joff.begin(), joff.end()), rl(row_l.begin(), row_l.end()), rm(row_m.begin(), row_m.end());
  jo.resize(7, 0);
  const at::cuda::CUDAGuard guard(vec.device());
  check(maloq::edge_rotation(vec.data_ptr<float>(), vec.stride(0), J.data_ptr<float>(), jo.data(), (int)L, rl.data(),
                             rm.data(), (int)rl.size(), ROT.data_ptr<float>(), (int)vec.size(0), stream()));
}

// Block <-> label rows fused with the block-diagonal basis transform (see labels.cu).
// data-side tensors (gather input / scatter output) are flat; rows are [rows, d].
void basis_rows(at::Tensor in, at::Tensor out, c10::optional<at::Tensor> ptr, c10::optional<at::Tensor> pt,
                c10::optional<at::Tensor> pos, at::Tensor meta, at::Tensor coef, int64_t d_in, int64_t rows,
                bool gather, bool scatter) {
  const auto dt = in.scalar_type();
  TORCH_CHECK(dt == at::kFloat || dt == at::kDouble, "basis_rows: fp32 or fp64");
  chk(in, dt, "in");
  chk(out, dt, "out");
  chk(coef, dt, "coef");
  chk(meta, at::kInt, "meta");
  TORCH_CHECK(meta.dim() == 2 && meta.size(1) == 4, "basis_rows: meta [d_out, 4]");
  maloq::BasisRowsArgs a{};
  a.in = in.data_ptr();
  a.out = out.data_ptr();
  a.d_in = (int)d_in;
  a.d_out = (int)meta.size(0);
  a.ld_in = d_in;
  a.ld_out = a.d_out;
  a.rows = rows;
  a.gather = gather;
  a.scatter = scatter;
  a.dtype = dt == at::kDouble ? 1 : 0;
  a.meta = reinterpret_cast<const int4*>(meta.data_ptr<int>());
  a.coef = coef.data_ptr();
  if (gather || scatter) {
    TORCH_CHECK(ptr && pt && pos, "basis_rows: gather/scatter needs ptr, pt, pos");
    chk(*ptr, at::kLong, "ptr");
    chk(*pt, at::kLong, "pt");
    chk(*pos, at::kInt, "pos");
    TORCH_CHECK(ptr->numel() >= rows && pt->numel() >= rows, "basis_rows: ptr/pt cover the rows");
    a.ptr = ll(*ptr);
    a.pt = ll(*pt);
    a.pos = pos->data_ptr<int>();
    a.d_pos = (int)pos->size(1);
    a.n_pt = pos->size(0);
    a.n_data = gather ? in.numel() : out.numel();
    TORCH_CHECK(a.d_pos == (gather ? a.d_in : a.d_out), "basis_rows: position table width");
  }
  if (!gather) TORCH_CHECK(in.numel() >= rows * d_in, "basis_rows: input rows");
  if (!scatter) TORCH_CHECK(out.numel() >= rows * a.d_out, "basis_rows: output rows");
  const at::cuda::CUDAGuard guard(in.device());
  check(maloq::basis_rows(a, stream()));
}

// Device radius graph (see graph.cu).  grid = [lo0, lo1, lo2, ext0, ext1, ext2, cutoff] (fp64 host
// list), ncell / periodic 3 ints.  mode 0: cell ids of all atoms -> out_cell; 1: per-target counts;
// 2: fill src/vec from ptr.
maloq::RadiusGraphArgs rg_args(const at::Tensor& pos, const std::vector<double>& grid, const std::vector<int64_t>& ncell,
                               const std::vector<int64_t>& periodic) {
  chk(pos, at::kDouble, "pos");
  TORCH_CHECK(pos.dim() == 2 && pos.size(1) == 3, "radius_graph: pos [N, 3]");
  TORCH_CHECK(grid.size() == 7 && ncell.size() == 3 && periodic.size() == 3, "radius_graph: grid description");
  maloq::RadiusGraphArgs a{};
  a.pos = pos.data_ptr<double>();
  for (int d = 0; d < 3; ++d) {
    a.lo[d] = grid[d];
    a.ext[d] = grid[3 + d];
    a.ncell[d] = (int)ncell[d];
    a.periodic[d] = (int)periodic[d];
    TORCH_CHECK(a.ncell[d] >= 1, "radius_graph: ncell >= 1");
  }
  a.cutoff = grid[6];
  return a;
}

void radius_graph_cells(at::Tensor pos, std::vector<double> grid, std::vector<int64_t> ncell,
                        std::vector<int64_t> periodic, at::Tensor cell) {
  auto a = rg_args(pos, grid, ncell, periodic);
  chk(cell, at::kLong, "cell");
  TORCH_CHECK(cell.numel() == pos.size(0), "radius_graph_cells: one id per atom");
  const at::cuda::CUDAGuard guard(pos.device());
  check(maloq::radius_graph_cells(a, pos.size(0), reinterpret_cast<long long*>(cell.data_ptr<int64_t>()), stream()));
}

void radius_graph_pass(at::Tensor pos, std::vector<double> grid, std::vector<int64_t> ncell,
                       std::vector<int64_t> periodic, at::Tensor targets, at::Tensor sorted_atoms,
                       at::Tensor cell_start, c10::optional<at::Tensor> counts, c10::optional<at::Tensor> ptr_,
                       c10::optional<at::Tensor> src, c10::optional<at::Tensor> vec) {
  auto a = rg_args(pos, grid, ncell, periodic);
  chk(targets, at::kLong, "targets");
  chk(sorted_atoms, at::kLong, "sorted_atoms");
  chk(cell_start, at::kLong, "cell_start");
  TORCH_CHECK(cell_start.numel() == ncell[0] * ncell[1] * ncell[2] + 1, "radius_graph: cell_start [n_cells + 1]");
  a.targets = ll(targets);
  a.n_targets = (int)targets.numel();
  a.sorted_atoms = ll(sorted_atoms);
  a.cell_start = ll(cell_start);
  const bool fill = ptr_.has_value();
  if (fill) {
    TORCH_CHECK(src && vec, "radius_graph fill: src and vec outputs");
    chk(*ptr_, at::kLong, "ptr");
    chk(*src, at::kLong, "src");
    chk(*vec, at::kDouble, "vec");
    a.ptr = ll(*ptr_);
    a.src = reinterpret_cast<long long*>(src->data_ptr<int64_t>());
    a.vec = vec->data_ptr<double>();
  } else {
    TORCH_CHECK(counts.has_value(), "radius_graph count: counts output");
    chk(*counts, at::kLong, "counts");
    a.counts = reinterpret_cast<long long*>(counts->data_ptr<int64_t>());
  }
  const at::cuda::CUDAGuard guard(pos.device());
  check(maloq::radius_graph_pass(a, fill, stream()));
}

// OUT [E, 2C + NB] bf16: [src_table[src_z] | exp(coeff (d - offset)^2) | dst_table[dst_z]], d = column 0
// of the edge attributes [E, A]
void edge_inputs(at::Tensor src_z, at::Tensor dst_z, at::Tensor edge_attr, at::Tensor src_table, at::Tensor dst_table,
                 at::Tensor offset, double coeff, at::Tensor OUT) {
  chk(src_z, at::kLong, "src_z");
  chk(dst_z, at::kLong, "dst_z");
  chk(edge_attr, at::kFloat, "edge_attr");
  chk(src_table, at::kFloat, "src_table");
  chk(dst_table, at::kFloat, "dst_table");
  chk(offset, at::kFloat, "offset");
  chk(OUT, at::kBFloat16, "OUT");
  const int64_t E = src_z.numel(), C = src_table.size(1), NB = offset.numel();
  TORCH_CHECK(dst_z.numel() == E && edge_attr.dim() == 2 && edge_attr.size(0) == E, "edge_inputs: edge counts");
  TORCH_CHECK(dst_table.sizes() == src_table.sizes(), "edge_inputs: tables of one shape");
  TORCH_CHECK(OUT.dim() == 2 && OUT.size(0) == E && OUT.size(1) == 2 * C + NB, "edge_inputs: OUT [E, 2C + NB]");
  const at::cuda::CUDAGuard guard(OUT.device());
  check(maloq::edge_inputs(ll(src_z), ll(dst_z), edge_attr.data_ptr<float>(), edge_attr.size(1),
                           src_table.data_ptr<float>(), dst_table.data_ptr<float>(), src_table.size(0),
                           offset.data_ptr<float>(), (float)coeff, bf(OUT), E, (int)C, (int)NB, stream()));
}

// out[N] (fp32, contiguous) = column sums of the 2-D X (fp32 or bf16, unit column stride, any
// row stride) in a fixed order; the partial-sum scratch comes from the caching allocator
void colsum(at::Tensor X, at::Tensor out) {
  TORCH_CHECK(X.is_cuda() && X.dim() == 2 && (X.scalar_type() == at::kFloat || X.scalar_type() == at::kBFloat16),
              "colsum: X must be a 2-D fp32 or bf16 CUDA tensor");
  TORCH_CHECK(X.size(1) <= 1 || X.stride(1) == 1, "colsum: X needs unit column stride");
  chk(out, at::kFloat, "colsum out");
  TORCH_CHECK(out.numel() == X.size(1), "colsum: out has one value per column");
  const long long M = X.size(0);
  const int N = (int)X.size(1);
  const int P = maloq::colsum_chunks(M, N);
  const at::cuda::CUDAGuard guard(X.device());
  at::Tensor part;
  if (P > 1) part = at::empty({P, (long long)N}, X.options().dtype(at::kFloat));
  check(maloq::colsum(X.data_ptr(), X.scalar_type() == at::kBFloat16, M, N, M > 1 ? X.stride(0) : (long long)N,
                      P > 1 ? part.data_ptr<float>() : nullptr, P, out.data_ptr<float>(), stream()));
}

// out[s] = column sums of rows [seg[s], seg[s + 1]) of the fp32 2-D X (unit column stride);
// out: contiguous fp32 holding len(seg) - 1 rows of X.size(1) values
void colsum_segments(at::Tensor X, std::vector<int64_t> seg, at::Tensor out) {
  TORCH_CHECK(X.is_cuda() && X.dim() == 2 && X.scalar_type() == at::kFloat, "colsum_segments: 2-D fp32 CUDA X");
  TORCH_CHECK(X.size(1) <= 1 || X.stride(1) == 1, "colsum_segments: X needs unit column stride");
  chk(out, at::kFloat, "colsum_segments out");
  TORCH_CHECK(seg.size() >= 2 && seg.front() >= 0 && seg.back() <= X.size(0), "colsum_segments: row offsets");
  TORCH_CHECK(out.numel() == (int64_t)(seg.size() - 1) * X.size(1), "colsum_segments: out size");
  std::vector<long long> s(seg.begin(), seg.end());
  const at::cuda::CUDAGuard guard(X.device());
  check(maloq::colsum_segments(X.data_ptr<float>(), (int)X.size(1), X.size(0) > 1 ? X.stride(0) : X.size(1), s.data(),
                               (int)s.size() - 1, out.data_ptr<float>(), stream()));
}

// Weight operand copies and pair-matrix gradients (kinds: maloq::kPack*), all jobs in one or a
// few launches.  srcs: contiguous fp32 CUDA tensors (1-D, 2-D or a 3-D batch of matrices).
void weight_pack(std::vector<at::Tensor> srcs, std::vector<at::Tensor> dsts, std::vector<int64_t> kinds) {
  const size_t n = srcs.size();
  TORCH_CHECK(dsts.size() == n && kinds.size() == n, "weight_pack: one destination and kind per source");
  if (n == 0) return;
  std::vector<const float*> sp(n);
  std::vector<void*> dp(n);
  std::vector<int> batch(n), rows(n), cols(n), kind(n);
  for (size_t g = 0; g < n; ++g) {
    const at::Tensor& S = srcs[g];
    const at::Tensor& D = dsts[g];
    chk(S, at::kFloat, "weight_pack source");
    TORCH_CHECK(S.device() == srcs[0].device() && D.device() == S.device(), "weight_pack: one device");
    TORCH_CHECK(S.dim() >= 1 && S.dim() <= 3, "weight_pack: 1-D, 2-D or 3-D sources");
    batch[g] = S.dim() == 3 ? (int)S.size(0) : 1;
    rows[g] = S.dim() >= 2 ? (int)S.size(S.dim() - 2) : 1;
    cols[g] = (int)S.size(S.dim() - 1);
    kind[g] = (int)kinds[g];
    const bool grad = kind[g] == maloq::kPackPairGrad;
    const bool pair = kind[g] == maloq::kPackPair || kind[g] == maloq::kPackPairT;
    chk(D, grad ? at::kFloat : at::kBFloat16, "weight_pack destination");
    TORCH_CHECK(D.numel() == (pair ? 2 * S.numel() : (grad ? S.numel() / 2 : S.numel())),
                "weight_pack: destination size does not match the job");
    sp[g] = S.data_ptr<float>();
    dp[g] = D.data_ptr();
  }
  const at::cuda::CUDAGuard guard(srcs[0].device());
  check(maloq::weight_pack((int)n, sp.data(), dp.data(), batch.data(), rows.data(), cols.data(), kind.data(),
                           stream()));
}

int64_t fock_loss_grid(int64_t n) { return maloq::fock_loss_grid(n); }

void fock_loss_stats(at::Tensor O, at::Tensor T, at::Tensor pt, at::Tensor mask, at::Tensor part) {
  chk(O, at::kFloat, "output");
  chk(T, at::kFloat, "target");
  chk(mask, at::kByte, "mask");
  chk(part, at::kFloat, "part");
  const at::cuda::CUDAGuard guard(O.device());
  check(maloq::fock_loss_stats(O.data_ptr<float>(), T.data_ptr<float>(), ll(pt), mask.data_ptr<uint8_t>(),
                               (int)O.size(1), O.size(0), part.data_ptr<float>(), (int)part.size(0), mask.size(0),
                               stream()));
}

// G = d(loss)/d(O) from gstat[0] = d/d(sse), gstat[1] = d/d(sae) (device tensor, any offset)
void fock_loss_grad(at::Tensor O, at::Tensor T, at::Tensor pt, at::Tensor mask, at::Tensor gstat, at::Tensor G) {
  chk(O, at::kFloat, "output");
  chk(G, at::kFloat, "grad");
  TORCH_CHECK(gstat.is_cuda() && gstat.scalar_type() == at::kFloat && gstat.numel() >= 2 && gstat.stride(0) == 1,
              "fock_loss_grad: gstat needs 2 contiguous fp32 values on the device");
  const at::cuda::CUDAGuard guard(O.device());
  check(maloq::fock_loss_grad(O.data_ptr<float>(), T.data_ptr<float>(), ll(pt), mask.data_ptr<uint8_t>(),
                              (int)O.size(1), O.size(0), gstat.data_ptr<float>(), G.data_ptr<float>(), mask.size(0),
                              stream()));
}

int64_t error_status(bool clear) { return maloq::error_status(clear); }
bool bounds_checked() { return maloq::bounds_checked(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &gemm, "grouped tcgen05 bf16 GEMM", py::arg("As"), py::arg("Bs"), py::arg("Cs"), py::arg("biases"),
        py::arg("mn_major"), py::arg("act"), py::arg("alpha"), py::arg("splits"), py::arg("bn"),
        py::arg("resids") = std::vector<c10::optional<at::Tensor>>());
  m.def("splitk_reduce", &splitk_reduce, "sum split-K partials");
  m.def("gather_rotate_fwd", &gather_rotate_fwd);
  m.def("gather_rotate_bwd", &gather_rotate_bwd, py::arg("L"), py::arg("MM"), py::arg("X"), py::arg("XE"),
        py::arg("rot"), py::arg("rad"), py::arg("dA"), py::arg("dst_ptr"), py::arg("src_perm"), py::arg("src_ptr"),
        py::arg("DX"), py::arg("DXE"), py::arg("DRAD"), py::arg("Cin"), py::arg("peers"), py::arg("halo_owner"),
        py::arg("halo_row"), py::arg("n_own"), py::arg("recv") = 0, py::arg("recv_slot") = py::none());
  m.def("rotate_back_scatter", &rotate_back_scatter);
  m.def("rotate_back_edge", &rotate_back_edge);
  m.def("rotate_grad", &rotate_grad);
  m.def("gate_fwd", &gate_fwd);
  m.def("gate_bwd", &gate_bwd);
  m.def("node_reduce", &node_reduce);
  m.def("halo_push", &halo_push);
  m.def("halo_fetch", &halo_fetch);
  m.def("rms_norm_fwd", &rms_norm_fwd);
  m.def("rms_norm_bwd", &rms_norm_bwd);
  m.def("norm_grid", &norm_grid);
  m.def("ln_silu_fwd", &ln_silu_fwd);
  m.def("ln_silu_bwd", &ln_silu_bwd);
  m.def("gate_l_fwd", &gate_l_fwd, py::arg("L"), py::arg("X"), py::arg("Gt"), py::arg("OUT"),
        py::arg("silu_gates") = false);
  m.def("gate_l_bwd", &gate_l_bwd, py::arg("L"), py::arg("X"), py::arg("Gt"), py::arg("DO"), py::arg("DX"),
        py::arg("DG"), py::arg("silu_gates") = false);
  m.def("head_gate_fwd", &head_gate_fwd);
  m.def("head_gate_bwd", &head_gate_bwd);
  m.def("edge_inputs", &edge_inputs);
  m.def("peer_barrier", &peer_barrier);
  m.def("peer_barrier_mask", &peer_barrier_mask);
  m.def("allreduce_p2p", &allreduce_p2p);
  m.def("allreduce_multimem", &allreduce_multimem);
  m.def("edge_rotation", &edge_rotation);
  m.def("fock_loss_grid", &fock_loss_grid);
  m.def("colsum", &colsum, "fixed-order column sums (fp32 out)");
  m.def("colsum_segments", &colsum_segments, "fixed-order column sums of row segments");
  m.def("weight_pack", &weight_pack, "bf16 weight operand copies / pair-matrix gradients in one launch");
  m.def("fock_loss_stats", &fock_loss_stats);
  m.def("basis_rows", &basis_rows);
  m.def("radius_graph_cells", &radius_graph_cells);
  m.def("radius_graph_pass", &radius_graph_pass);
  m.def("fock_loss_grad", &fock_loss_grad);
  m.def("error_status", &error_status, "read/clear the device error word", py::arg("clear") = true);
  m.def("bounds_checked", &bounds_checked, "true for a library built with device index checks");
}
