"""tcgen05 GEMM kernel vs an fp32 PyTorch reference of the same bf16-rounded operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _k():
    from maloq_b200.ops import kernels

    return kernels


def _ref(a, w, bias=None):
    y = a.to(torch.bfloat16).float() @ w.to(torch.bfloat16).float().t()
    return y if bias is None else y + bias


def _close(out, ref, tol=2e-3):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, (err, scale)


@pytest.mark.parametrize("M,N,K,bn", [(128, 128, 64, 128), (300, 72, 136, 64), (1000, 1152, 1280, 256),
                                      (4096, 1024, 1024, 128), (77, 200, 520, 256), (513, 640, 384, 128)])
def test_gemm_nt_shapes(cuda_device, M, N, K, bn):
    k = _k()
    torch.manual_seed(0)
    a = torch.randn(M, K, device=cuda_device)
    w = torch.randn(N, K, device=cuda_device) / K ** 0.5
    b = torch.randn(N, device=cuda_device)
    out = k.gemm_nt(a, w, b, bn=bn)
    _close(out, _ref(a, w, b))
    assert k.error_status() == 0


def test_gemm_bf16_out_and_silu(cuda_device):
    k = _k()
    a = torch.randn(640, 256, device=cuda_device)
    w = torch.randn(384, 256, device=cuda_device) / 16
    out = k.gemm_nt(a, w, out_dtype=torch.bfloat16, act=1)
    _close(out, torch.nn.functional.silu(_ref(a, w)), tol=1e-2)


def test_gemm_grouped(cuda_device):
    k = _k()
    lib = k.lib()
    shapes = [(700, 1152, 1280), (700, 1024, 1024), (700, 768, 768)]
    As = [torch.randn(m, kk, device=cuda_device).bfloat16() for m, n, kk in shapes]
    Ws = [(torch.randn(n, kk, device=cuda_device) / kk ** 0.5).bfloat16() for m, n, kk in shapes]
    Cs = [torch.empty(m, n, device=cuda_device) for m, n, kk in shapes]
    lib.gemm(As, Ws, Cs, [None, None, None], False, 0, 1.0, 1, 128)
    for A, W, C in zip(As, Ws, Cs):
        _close(C, A.float() @ W.float().t())


@pytest.mark.parametrize("M,N,K", [(43000, 1152, 1280), (1000, 72, 136), (333, 128, 128)])
def test_weight_grad_splitk_deterministic(cuda_device, M, N, K):
    k = _k()
    torch.manual_seed(1)
    gy = torch.randn(M, N, device=cuda_device)
    x = torch.randn(M, K, device=cuda_device)
    dw = k.gemm_tn_weight_grad(gy, x)
    ref = gy.bfloat16().float().t() @ x.bfloat16().float()
    _close(dw, ref)
    assert torch.equal(dw, k.gemm_tn_weight_grad(gy, x))


def test_linear_autograd_matches_torch(cuda_device):
    from maloq_b200 import ops

    torch.manual_seed(2)
    x = torch.randn(900, 192, device=cuda_device, requires_grad=True)
    w = torch.randn(320, 192, device=cuda_device, requires_grad=True)
    b = torch.randn(320, device=cuda_device, requires_grad=True)
    y = ops.linear(x, w, b, act="silu")
    g = torch.randn_like(y)
    (y * g).sum().backward()
    x2, w2, b2 = (t.detach().bfloat16().float().requires_grad_() for t in (x, w, b))
    y2 = torch.nn.functional.silu(x2 @ w2.t() + b2)
    (y2 * g).sum().backward()
    _close(y, y2, 1e-2)
    _close(x.grad, x2.grad, 1e-2)
    _close(w.grad, w2.grad, 1e-2)
    _close(b.grad, b2.grad, 1e-3)


def test_linear_odd_sizes(cuda_device):
    from maloq_b200 import ops

    x = torch.randn(50, 13, device=cuda_device, requires_grad=True)
    w = torch.randn(7, 13, device=cuda_device, requires_grad=True)
    y = ops.linear(x, w)
    y.sum().backward()
    assert w.grad.shape == w.shape and x.grad.shape == x.shape
    _close(y, _ref(x.detach(), w.detach()), 1e-2)
