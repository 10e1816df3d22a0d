"""CUDA kernels whose source also builds as host C++ (no shared memory, warp intrinsics or
synchronisation), run over an emulated grid on the CPU and compared with PyTorch.  This checks
the kernels' own index arithmetic and math without a GPU; the GPU tests check the same kernels on
the device."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from tests.cpu_extension import CpuExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "maloq_b200", "ops", "csrc")
CUDA_INC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")


@pytest.fixture(scope="module")
def emu(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None or not os.path.isfile(os.path.join(CUDA_INC, "cuda_bf16.h")):
        pytest.skip("needs g++ and the CUDA headers")
    so = str(tmp_path_factory.mktemp("emu") / "head_gate_emu.so")
    subprocess.run([cxx, "-O1", "-std=c++17", "-shared", "-fPIC", "-I", CSRC, "-I", CUDA_INC,
                    os.path.join(HERE, "csrc", "head_gate_emu.cpp"), "-o", so], check=True)
    return ctypes.CDLL(so)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _gate_ref(x, sv, act, scale, absg):
    """The Fock head's gated operand (ops/reference.py fock_head_process, before the per-degree
    linears): row 0 the transformed scalars, every l >= 1 coefficient times its gate."""
    N, S, C = x.shape
    L = int(round(S ** 0.5)) - 1
    t0, g = sv[:, :C], sv[:, C:]
    if absg:
        g = g.abs()
    g = (torch.sigmoid(g) if act == 0 else torch.tanh(g)) * scale
    g = g.view(N, L, C)
    rows = [t0.unsqueeze(1)]
    for l in range(1, L + 1):
        rows.append(x[:, l * l:(l + 1) ** 2] * g[:, l - 1].unsqueeze(1))
    return torch.cat(rows, dim=1)


@pytest.mark.parametrize("L,C,act,absg", [(0, 8, 0, False), (1, 5, 1, True), (2, 128, 0, True), (4, 128, 1, False),
                                          (4, 33, 0, False), (6, 16, 1, True)])
@pytest.mark.parametrize("grid", [1, 3, 64])
def test_head_gate_kernels_on_emulated_grid(emu, L, C, act, absg, grid):
    torch.manual_seed(L * 100 + C + grid)
    N, S = 7, (L + 1) ** 2
    scale = 1.7
    x = torch.randn(N, S, C, dtype=torch.float32, requires_grad=True)
    sv = torch.randn(N, (L + 1) * C, dtype=torch.float32, requires_grad=True)
    with torch.no_grad():
        sv[0, C:C + 3] = 0.0  # |u| at u = 0: zero gradient, as PyTorch's abs
    A = torch.empty(N, S, C, dtype=torch.bfloat16)
    assert emu.emu_head_gate_fwd(L, _p(x), _p(sv), _p(A), act, ctypes.c_float(scale), int(absg), N, C, grid, 32) == 0
    ref = _gate_ref(x, sv, act, scale, absg)
    # bf16 rounding of the same fp32 value; the host's tanhf / expf may differ from PyTorch's by
    # an ulp, which can move a value across a bf16 rounding boundary (one bf16 ulp: 2^-8 relative)
    r = ref.detach()
    np.testing.assert_allclose(A.float().numpy(), r.numpy(), rtol=2 ** -8, atol=1e-30)
    assert (A != r.to(torch.bfloat16)).float().mean().item() < 0.01
    dA = torch.randn(N, S, C)
    dx, dsv = torch.full_like(x, float("nan")), torch.full_like(sv, float("nan"))
    assert emu.emu_head_gate_bwd(L, _p(x), _p(sv), _p(dA), _p(dx), _p(dsv), act, ctypes.c_float(scale), int(absg),
                                 N, C, grid, 32) == 0
    rdx, rdsv = torch.autograd.grad(ref, [x, sv], dA, allow_unused=True)
    rdx = torch.zeros_like(x) if rdx is None else rdx
    np.testing.assert_allclose(dx.numpy(), rdx.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dsv.numpy(), rdsv.numpy(), rtol=1e-5, atol=1e-6)


class _CpuExtension(CpuExtension):
    """The CPU stand-in of the extension with the head-gate calls running the kernel source
    on the emulated grid."""

    def __init__(self, emu):
        self.emu = emu

    def head_gate_fwd(self, L, x, sv, A, act, scale, absg):
        N, S, C = x.shape
        assert self.emu.emu_head_gate_fwd(L, _p(x), _p(sv), _p(A), act, ctypes.c_float(scale), int(absg), N, C,
                                          max(1, min((N * C + 255) // 256, 148 * 32)), 256) == 0

    def head_gate_bwd(self, L, x, sv, dA, dx, dsv, act, scale, absg):
        N, S, C = x.shape
        assert self.emu.emu_head_gate_bwd(L, _p(x), _p(sv), _p(dA), _p(dx), _p(dsv), act, ctypes.c_float(scale),
                                          int(absg), N, C, max(1, min((N * C + 255) // 256, 148 * 32)), 256) == 0


@pytest.mark.parametrize("act,absg,muls", [("sigmoid", False, [3, 0, 5, 2, 1]), ("tanh", True, [9, 4, 0, 11, 6])])
def test_fock_head_kernel_path_on_cpu(emu, monkeypatch, act, absg, muls):
    """The kernel path of the Fock head's process step (head_gate + per-coefficient grouped GEMMs
    + sorted-order gather, and its backward) against the PyTorch definition, with bf16 GEMM
    operands emulated on the CPU."""
    from maloq_b200.ops import kernels
    from maloq_b200.ops import reference as R

    monkeypatch.setattr(kernels, "_lib", _CpuExtension(emu))
    torch.manual_seed(3)
    L, C, N = 4, 16, 37
    S = (L + 1) ** 2
    x = torch.randn(N, S, C, requires_grad=True)
    ws = torch.nn.Parameter(torch.randn((L + 1) * C, C) / C ** 0.5)
    bs = torch.nn.Parameter(torch.randn((L + 1) * C) * 0.1)
    layers = []
    for l, m in enumerate(muls):
        if m == 0:
            layers.append((None, None))
            continue
        w = torch.nn.Parameter(torch.randn(m, C) / C ** 0.5)
        b = torch.nn.Parameter(torch.randn(m) * 0.1) if l == 0 else None
        layers.append((w, b))
    params = [x, ws, bs] + [t for wb in layers for t in wb if t is not None]
    out = kernels._head_process(x, ws, bs, layers, act, 1.3, absg)
    ref = R.fock_head_process(x, ws, bs, layers, act, 1.3, absg)
    assert out.shape == ref.shape == (N, sum(m * (2 * l + 1) for l, m in enumerate(muls)))
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()
    assert rel(out, ref) < 1e-2  # bf16 GEMM operands
    g = torch.randn_like(ref)
    got = torch.autograd.grad((out * g).sum(), params)
    want = torch.autograd.grad((ref * g).sum(), params)
    for a, b in zip(got, want):
        assert a.shape == b.shape
        assert rel(a, b) < 2e-2, rel(a, b)


def test_weight_cache_layouts_and_refresh():
    """bf16 copies of the GEMM weights (plain, transposed, SO(2) pair form and its transpose)
    match their definitions and are rebuilt after an optimizer step changes the parameter."""
    from maloq_b200.ops import weights as W

    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(8, 6))
    q = torch.nn.Parameter(torch.randn(3, 4, 5))
    opt = torch.optim.SGD([p, q], lr=0.1)
    for _ in range(2):
        wr, wi = p.detach()[:4], p.detach()[4:]
        pair = torch.cat([torch.cat([wr, -wi], 1), torch.cat([wi, wr], 1)], 0)
        assert torch.equal(W.pair_bf16(p), pair.bfloat16())
        assert torch.equal(W.pair_bf16_t(p), pair.t().bfloat16())
        assert torch.equal(W.bf16(p), p.detach().bfloat16())
        assert torch.equal(W.bf16_t(q), q.detach().transpose(-1, -2).bfloat16())
        dP = torch.randn(8, 12)
        g = W.pair_grad(dP)
        pr = p.detach().clone().requires_grad_()
        wr_, wi_ = pr[:4], pr[4:]
        (torch.cat([torch.cat([wr_, -wi_], 1), torch.cat([wi_, wr_], 1)], 0) * dP).sum().backward()
        assert torch.allclose(g, pr.grad)
        (p.sum() + q.sum()).backward()
        opt.step()
        opt.zero_grad()


def test_weight_cache_entries_die_with_their_parameter():
    """A cached bf16 copy is dropped when its parameter is freed, so a new parameter that reuses
    the freed one's id and storage address cannot be served the old copy."""
    import gc

    from maloq_b200.ops import weights as W

    p = torch.nn.Parameter(torch.randn(4, 4))
    W.bf16(p)
    key = (id(p), "bf16")
    assert key in W._CACHE and W._CACHE[key][2]() is p
    del p
    gc.collect()
    assert key not in W._CACHE


@pytest.mark.parametrize("E,C,NB,grid", [(37, 16, 8, 1), (200, 128, 128, 7), (5, 8, 3, 64)])
def test_edge_inputs_kernel_on_emulated_grid(tmp_path, E, C, NB, grid):
    """The radial-input kernel (embedding rows around the Gaussian expansion of the edge length,
    bf16) from its own source on an emulated grid against PyTorch; an element index outside the
    table is zeroed and reported."""
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("needs g++")
    so = str(tmp_path / "ei.so")
    subprocess.run([cxx, "-O1", "-std=c++17", "-shared", "-fPIC", "-I", CSRC, "-I", CUDA_INC,
                    os.path.join(HERE, "csrc", "edge_inputs_emu.cpp"), "-o", so], check=True)
    lib = ctypes.CDLL(so)
    torch.manual_seed(E)
    V = 12
    src_z, dst_z = torch.randint(0, V, (E,)), torch.randint(0, V, (E,))
    attr = torch.rand(E, 4) * 6
    st, dt = torch.randn(V, C), torch.randn(V, C)
    off = torch.linspace(0, 6, NB)
    coeff = -0.5 / float(off[1] - off[0]) ** 2 if NB > 1 else -1.0
    out = torch.empty(E, 2 * C + NB, dtype=torch.bfloat16)
    err = lib.emu_edge_inputs(_p(src_z), _p(dst_z), _p(attr), ctypes.c_longlong(4), _p(st), _p(dt),
                              ctypes.c_longlong(V), _p(off), ctypes.c_float(coeff), _p(out), ctypes.c_longlong(E), C, NB,
                              grid, 64)
    assert err == 0
    ref = torch.cat([st[src_z], torch.exp(coeff * (attr[:, :1] - off.view(1, -1)) ** 2), dt[dst_z]], 1)
    np.testing.assert_allclose(out.float().numpy(), ref.numpy(), rtol=2 ** -8, atol=1e-30)
    bad = src_z.clone()
    bad[0] = V
    err = lib.emu_edge_inputs(_p(bad), _p(dst_z), _p(attr), ctypes.c_longlong(4), _p(st), _p(dt),
                              ctypes.c_longlong(V), _p(off), ctypes.c_float(coeff), _p(out), ctypes.c_longlong(E), C, NB,
                              grid, 64)
    assert err == 5 and torch.all(out[0, :C] == 0)
