"""Norm / gate / SO3-linear kernels vs their fp32 PyTorch definitions (forward + grads)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-12)).item()


def _balance(L, dev):
    bw = torch.zeros((L + 1) ** 2, 1, device=dev)
    for l in range(L + 1):
        bw[l * l:(l + 1) ** 2] = 1.0 / (2 * l + 1)
    return bw / (L + 1)


@pytest.mark.parametrize("L,C,res", [(4, 128, False), (4, 128, True), (2, 32, True), (6, 64, False)])
def test_rms_norm(cuda_device, L, C, res):
    from maloq_b200.ops import norm_native
    from maloq_b200.ops import reference as R

    torch.manual_seed(0)
    B, S = 300, (L + 1) ** 2
    x = torch.randn(B, S, C, device=cuda_device, requires_grad=True)
    r = torch.randn(B, S, C, device=cuda_device, requires_grad=True) if res else None
    aw = (1 + 0.1 * torch.randn(L + 1, C, device=cuda_device)).requires_grad_()
    ab = (0.1 * torch.randn(C, device=cuda_device)).requires_grad_()
    args = [x, aw, ab] + ([r] if res else [])
    out = norm_native.rms_norm_sh(x, aw, ab, 1e-5, r)
    ref = R.rms_norm_sh(x, aw, ab, _balance(L, cuda_device), 1e-5, r)
    if res:
        g1, g2 = torch.randn_like(out[0]), torch.randn_like(out[1])
        loss, rloss = (out[0] * g1).sum() + (out[1] * g2).sum(), (ref[0] * g1).sum() + (ref[1] * g2).sum()
        assert _rel(out[0], ref[0]) < 1e-5 and _rel(out[1], ref[1]) < 1e-6
    else:
        g1 = torch.randn_like(out)
        loss, rloss = (out * g1).sum(), (ref * g1).sum()
        assert _rel(out, ref) < 1e-5
    for a, b in zip(torch.autograd.grad(loss, args), torch.autograd.grad(rloss, args)):
        assert _rel(a, b) < 1e-4


def test_layernorm_silu(cuda_device):
    from maloq_b200.ops import norm_native

    x = torch.randn(5000, 128, device=cuda_device, requires_grad=True)
    w = (1 + 0.1 * torch.randn(128, device=cuda_device)).requires_grad_()
    b = (0.1 * torch.randn(128, device=cuda_device)).requires_grad_()
    out = norm_native.layernorm_silu(x, w, b)
    ref = torch.nn.functional.silu(torch.nn.functional.layer_norm(x, (128,), w, b, 1e-5))
    assert out.dtype == torch.bfloat16 and _rel(out, ref) < 1e-2
    g = torch.randn_like(ref).bfloat16().float()
    ga = torch.autograd.grad((out.float() * g).sum(), [x, w, b])
    gr = torch.autograd.grad((ref * g).sum(), [x, w, b])
    for a, bb in zip(ga, gr):
        assert _rel(a, bb) < 1e-4


def test_gate_l(cuda_device):
    from maloq_b200.ops import norm_native
    from maloq_b200.ops import reference as R

    L, H = 4, 64
    x = torch.randn(200, 25, H, device=cuda_device, requires_grad=True)
    g = torch.randn(200, L * H, device=cuda_device, requires_grad=True)
    idx = torch.cat([torch.full((2 * l + 1,), l - 1) for l in range(1, L + 1)]).to(cuda_device)
    out = norm_native.gate_l(g, x, L)
    ref = R.gate(g, x, idx, L)
    assert _rel(out, ref) < 1e-6
    w = torch.randn_like(out)
    for a, b in zip(torch.autograd.grad((out * w).sum(), [g, x]), torch.autograd.grad((ref * w).sum(), [g, x])):
        assert _rel(a, b) < 1e-5


def test_gate_with_silu_gates(cuda_device):
    """Gate fed the pre-activations (SiLU inside the kernels) vs gate(silu(pre), x) in fp32."""
    from maloq_b200.ops import norm_native
    from maloq_b200.ops import reference as R

    L, H = 4, 64
    x = torch.randn(200, 25, H, device=cuda_device, requires_grad=True)
    pre = (2 * torch.randn(200, L * H, device=cuda_device)).requires_grad_()
    idx = torch.cat([torch.full((2 * l + 1,), l - 1) for l in range(1, L + 1)]).to(cuda_device)
    out = norm_native.gate_l(pre, x, L, silu_gates=True)
    ref = R.gate(torch.nn.functional.silu(pre), x, idx, L)
    assert _rel(out, ref) < 1e-6
    w = torch.randn_like(out)
    for a, b in zip(torch.autograd.grad((out * w).sum(), [pre, x]), torch.autograd.grad((ref * w).sum(), [pre, x])):
        assert _rel(a, b) < 1e-5


def test_so3_linear(cuda_device):
    from maloq_b200.ops import norm_native
    from maloq_b200.ops import reference as R

    torch.manual_seed(0)
    x = torch.randn(3000, 25, 128, device=cuda_device, requires_grad=True)
    W = (torch.randn(5, 96, 128, device=cuda_device) / 11).requires_grad_()
    b = torch.randn(96, device=cuda_device, requires_grad=True)
    out = norm_native.so3_linear(x, W, b, 4)
    ref = R.so3_linear(x.bfloat16().float(), W.bfloat16().float(), b, 4)
    assert _rel(out, ref) < 2e-3
    g = torch.randn_like(out)
    ga = torch.autograd.grad((out * g).sum(), [x, W, b])
    gr = torch.autograd.grad((R.so3_linear(x, W, b, 4) * g).sum(), [x, W, b])
    for a, bb in zip(ga, gr):
        assert _rel(a, bb) < 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_so3_linear_with_scalar_side_linear(cuda_device, dtype):
    """The atomwise block's SO3 linear and its gate-scalar linear of x[:, 0] as one autograd node
    (the scalar linear's input gradient added into row 0 in place) vs the two separate ops."""
    from maloq_b200.ops import norm_native
    from maloq_b200.ops import reference as R

    torch.manual_seed(1)
    x = torch.randn(2000, 25, 128, device=cuda_device).to(dtype).requires_grad_()
    W = (torch.randn(5, 128, 128, device=cuda_device) / 11).requires_grad_()
    b = torch.randn(128, device=cuda_device, requires_grad=True)
    sw = (torch.randn(512, 128, device=cuda_device) / 11).requires_grad_()
    sb = torch.randn(512, device=cuda_device, requires_grad=True)
    h, pre = norm_native.so3_linear_scalar(x, W, b, 4, torch.bfloat16, sw, sb)
    assert h.dtype == torch.bfloat16 and pre.dtype == torch.float32
    xf = x.float()
    rh, rp = R.so3_linear(xf, W, b, 4), R.linear(xf[:, 0], sw, sb)
    assert _rel(h, rh) < 1e-2 and _rel(pre, rp) < 1e-2
    gh, gp = torch.randn_like(rh), torch.randn_like(rp)
    got = torch.autograd.grad((h.float() * gh).sum() + (pre * gp).sum(), [x, W, b, sw, sb])
    want = torch.autograd.grad((rh * gh).sum() + (rp * gp).sum(), [x, W, b, sw, sb])
    for a, r in zip(got, want):
        assert a.dtype == r.dtype or a.dtype == dtype
        assert ((a.float() - r.float()).norm() / r.float().norm()).item() < 1.5e-2


@pytest.mark.parametrize("act,absg,muls,N", [("sigmoid", False, [14, 0, 9, 3, 1], 700),
                                             ("tanh", True, [14, 10, 9, 3, 1], 5000)])
def test_fock_head_process_kernel(cuda_device, act, absg, muls, N):
    """Fock head process step on the kernel path (head_gate + per-coefficient grouped GEMMs +
    sorted-order gather) vs its fp32 PyTorch definition, forward and gradients."""
    from maloq_b200.ops import kernels
    from maloq_b200.ops import reference as R

    torch.manual_seed(5)
    L, C = 4, 128
    S = (L + 1) ** 2
    dev = cuda_device
    x = torch.randn(N, S, C, device=dev, requires_grad=True)
    ws = torch.nn.Parameter(torch.randn((L + 1) * C, C, device=dev) / C ** 0.5)
    bs = torch.nn.Parameter(torch.randn((L + 1) * C, device=dev) * 0.1)
    layers = []
    for l, m in enumerate(muls):
        if m == 0:
            layers.append((None, None))
            continue
        w = torch.nn.Parameter(torch.randn(m, C, device=dev) / C ** 0.5)
        b = torch.nn.Parameter(torch.randn(m, device=dev) * 0.1) if l == 0 else None
        layers.append((w, b))
    params = [x, ws, bs] + [t for wb in layers for t in wb if t is not None]
    out = kernels._head_process(x, ws, bs, layers, act, 1.3, absg)
    ref = R.fock_head_process(x, ws, bs, layers, act, 1.3, absg)
    relf = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert out.shape == ref.shape
    assert relf(out, ref) < 1e-2, relf(out, ref)
    g = torch.randn_like(ref)
    got = torch.autograd.grad((out * g).sum(), params)
    want = torch.autograd.grad((ref * g).sum(), params)
    for a, b in zip(got, want):
        assert relf(a, b) < 1.5e-2, relf(a, b)
    assert kernels.error_status() == 0
