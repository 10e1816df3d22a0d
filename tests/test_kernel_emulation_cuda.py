"""The CUDA source of the edge-frame and normalisation kernels (ops/csrc/edge.cu, norm.cu), built
for the CPU with a small CUDA runtime emulator (tests/csrc/host_emu.cuh: one thread per CUDA
thread with real block barriers, emulated warp shuffles, alignment-checked vector loads) and run
through their own host launchers, against the contracts of the CPU stand-in
(tests/cpu_extension.py).  Small shapes; several (lmax, mmax) frames."""
import numpy as np
import pytest
import torch

from tests.cpu_extension import CpuExtension
from tests.emulated_extension import load_libraries

@pytest.fixture(scope="module")
def _libs(tmp_path_factory):
    libs = load_libraries(tmp_path_factory.mktemp("kernel_emu"), names=("edge", "norm"))
    if libs is None:
        pytest.skip("needs g++ and the CUDA headers")
    return libs


@pytest.fixture(scope="module")
def edge(_libs):
    return _libs["edge"]


@pytest.fixture(scope="module")
def norm(_libs):
    return _libs["norm"]


def _p(t):
    return None if t is None else t.data_ptr()


def _ok(r):
    assert r is None, r.decode()


def _close(a, b, rel=2 ** -7):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= rel * max(1.0, b.abs().max().item()), err


def _graph(N, E, seed):
    rng = np.random.default_rng(seed)
    dst = np.sort(rng.integers(0, N, E))
    src = rng.integers(0, N, E)
    dst_ptr = np.searchsorted(dst, np.arange(N + 1))
    perm = np.argsort(src, kind="stable")
    src_ptr = np.searchsorted(src[perm], np.arange(N + 1))
    t = lambda a: torch.as_tensor(a, dtype=torch.long)
    return t(src), t(dst), t(dst_ptr), t(perm), t(src_ptr)


FRAMES = [(4, 2), (2, 1), (3, 3), (6, 2)]


def _rot(E, L, MM, seed):
    from tests.cpu_extension import frame_rows

    ls, _, _ = frame_rows(L, MM)
    g = torch.Generator().manual_seed(seed)
    rot = torch.zeros(E, len(ls), (L + 1) ** 2)
    for k, l in enumerate(ls):  # only the row's degree block is non-zero
        rot[:, k, l * l:(l + 1) ** 2] = torch.randn(E, 2 * l + 1, generator=g)
    return rot


@pytest.mark.parametrize("L,MM", FRAMES)
@pytest.mark.parametrize("three", [False, True])
def test_gather_rotate_kernels(edge, L, MM, three):
    from tests.cpu_extension import frame_rows

    torch.manual_seed(L * 10 + MM)
    N, E, C = 9, 26, 8
    Cin = (3 if three else 2) * C
    S = (L + 1) ** 2
    ls, _, ns = frame_rows(L, MM)
    R = len(ls)
    src, dst, dptr, perm, sptr = _graph(N, E, L)
    X = torch.randn(N, S, C)
    XE = torch.randn(E, S, C) if three else None
    rot = _rot(E, L, MM, 1)
    rad = torch.randn(E, ns * Cin).to(torch.bfloat16)
    A = torch.empty(E, R * Cin, dtype=torch.bfloat16)
    _ok(edge.emu_gather_rotate_fwd(L, MM, _p(X), _p(XE), _p(src), _p(dst), _p(rot), _p(rad), _p(A), E, C, Cin, N))
    ref = CpuExtension()
    A2 = torch.empty_like(A)
    ref.gather_rotate_fwd(L, MM, X, XE, src, dst, rot, rad, A2, Cin, 0, None, None, 0)
    _close(A, A2)
    dA = torch.randn(E, R * Cin).to(torch.bfloat16)
    DX, DRAD = torch.full((N, S, C), float("nan")), torch.empty(E, ns * Cin, dtype=torch.bfloat16)
    DXE = torch.full((E, S, C), float("nan")) if three else None
    _ok(edge.emu_gather_rotate_bwd(L, MM, _p(X), _p(XE), _p(rot), _p(rad), _p(dA), _p(dptr), _p(perm), _p(sptr),
                                   _p(DX), _p(DXE), _p(DRAD), N, E, C, Cin))
    DX2, DRAD2 = torch.empty_like(DX), torch.empty_like(DRAD)
    DXE2 = torch.empty_like(DXE) if three else None
    ref.gather_rotate_bwd(L, MM, X, XE, rot, rad, dA, dptr, perm, sptr, DX2, DXE2, DRAD2, Cin)
    _close(DX, DX2, 1e-4)
    _close(DRAD, DRAD2)
    if three:
        _close(DXE, DXE2, 1e-4)
    assert edge.emu_error_word() == 0


@pytest.mark.parametrize("L,MM", FRAMES)
@pytest.mark.parametrize("C", [8, 6, 5])
def test_rotate_back_and_grad_kernels(edge, L, MM, C):
    from tests.cpu_extension import frame_rows

    torch.manual_seed(L + C)
    N, E = 7, 21
    S = (L + 1) ** 2
    R = len(frame_rows(L, MM)[0])
    _, dst, dptr, _, _ = _graph(N, E, C)
    rot = _rot(E, L, MM, 2)
    ldy, koff = R * C + 2 * C, 2 * C  # rows inside a wider buffer, as in the head / degree embedding
    Y = torch.randn(E, ldy).to(torch.bfloat16)
    ref = CpuExtension()
    for Rk in (R, L + 1):
        base = torch.randn(N, S, C)
        out, out2 = torch.empty(N, S, C), torch.empty(N, S, C)
        _ok(edge.emu_rotate_back_scatter(L, MM, _p(Y), ldy, koff, _p(rot), _p(dptr), _p(base), _p(out), N, C, Rk, 0.7))
        ref.rotate_back_scatter(L, MM, Y, koff, Rk, rot, dptr, base, out2, 0.7)
        _close(out, out2, 1e-4)
        oe, oe2 = torch.empty(E, S, C), torch.empty(E, S, C)
        _ok(edge.emu_rotate_back_edge(L, MM, _p(Y), ldy, koff, _p(rot), _p(oe), E, C, Rk))
        ref.rotate_back_edge(L, MM, Y, koff, Rk, rot, oe2)
        _close(oe, oe2, 1e-4)
        for rows in (dst, None):
            G = torch.randn(N if rows is not None else E, S, C)
            DY, DYf = torch.zeros(E, Rk * C, dtype=torch.bfloat16), torch.zeros(E, Rk * C)
            DY2, DYf2 = torch.zeros_like(DY), torch.zeros_like(DYf)
            _ok(edge.emu_rotate_grad(L, MM, _p(G), _p(rows), _p(rot), _p(DY), _p(DYf), E, C, Rk, 0.5))
            ref.rotate_grad(L, MM, G, rows, rot, DY2, DYf2, Rk, 0.5)
            _close(DYf, DYf2, 1e-4)
            _close(DY, DY2)


@pytest.mark.parametrize("L,MM", FRAMES)
def test_m_major_gate_kernels(edge, L, MM):
    from tests.cpu_extension import frame_rows

    torch.manual_seed(L)
    E, H = 13, 24
    R = len(frame_rows(L, MM)[0])
    Y1 = torch.randn(E, L * H + R * H).to(torch.bfloat16)
    H1, H1r = torch.empty(E, R * H, dtype=torch.bfloat16), torch.empty(E, R * H, dtype=torch.bfloat16)
    _ok(edge.emu_gate_fwd(L, MM, _p(Y1), _p(H1), E, H))
    ref = CpuExtension()
    ref.gate_fwd(L, MM, Y1, H1r, H)
    _close(H1, H1r)
    dH1 = torch.randn(E, R * H).to(torch.bfloat16)
    dY1, dY1r = torch.empty_like(Y1), torch.empty_like(Y1)
    _ok(edge.emu_gate_bwd(L, MM, _p(Y1), _p(dH1), _p(dY1), E, H))
    ref.gate_bwd(L, MM, Y1, dH1, dY1r, H)
    _close(dY1, dY1r)


@pytest.mark.parametrize("L,C", [(4, 128), (2, 64), (6, 32)])
@pytest.mark.parametrize("res,bf16", [(False, False), (True, True), (True, False)])
def test_rms_norm_kernels(norm, L, C, res, bf16):
    torch.manual_seed(L + C)
    B, S = 5, (L + 1) ** 2
    X = torch.randn(B, S, C)
    RES = torch.randn(B, S, C) if res else None
    aw, ab = 1 + 0.1 * torch.randn(L + 1, C), 0.1 * torch.randn(C)
    od = torch.bfloat16 if bf16 else torch.float32
    out, out2 = torch.empty(B, S, C, dtype=od), torch.empty(B, S, C, dtype=od)
    SUM, SUM2 = (torch.empty(B, S, C), torch.empty(B, S, C)) if res else (None, None)
    _ok(norm.emu_rms_norm_fwd(L, _p(X), _p(RES), _p(aw), _p(ab), _p(out), int(bf16), _p(SUM), B, C, 1e-6))
    ref = CpuExtension()
    ref.rms_norm_fwd(L, X, RES, aw, ab, out2, SUM2, 1e-6)
    _close(out, out2, 2 ** -7 if bf16 else 1e-4)
    s = SUM if res else X
    G = torch.randn(B, S, C).to(od)
    GS = torch.randn(B, S, C) if res else None
    grid = norm.emu_norm_grid(B)
    DX, PART = torch.empty(B, S, C), torch.empty(grid, L + 2, C)
    _ok(norm.emu_rms_norm_bwd(L, _p(s), _p(G), int(bf16), _p(GS), _p(aw), _p(DX), _p(PART), B, C, 1e-6, grid))
    DX2, PART2 = torch.empty(B, S, C), torch.empty(1, L + 2, C)
    ref.rms_norm_bwd(L, s, G, GS, aw, DX2, PART2, 1e-6)
    _close(DX, DX2, 1e-4)
    _close(PART.sum(0), PART2[0], 1e-4)


@pytest.mark.parametrize("W", [128, 384, 40])
def test_layernorm_silu_kernels(norm, W):
    torch.manual_seed(W)
    M = 37
    X, w, b = torch.randn(M, W), 1 + 0.1 * torch.randn(W), 0.1 * torch.randn(W)
    out, out2 = torch.empty(M, W, dtype=torch.bfloat16), torch.empty(M, W, dtype=torch.bfloat16)
    _ok(norm.emu_ln_silu_fwd(_p(X), _p(w), _p(b), _p(out), M, W, 1e-5))
    ref = CpuExtension()
    ref.ln_silu_fwd(X, w, b, out2, 1e-5)
    _close(out, out2)
    G = torch.randn(M, W).to(torch.bfloat16)
    grid = 3
    DX, PART = torch.empty(M, W), torch.empty(grid * 8, 2, W)
    _ok(norm.emu_ln_silu_bwd(_p(X), _p(w), _p(b), _p(G), _p(DX), _p(PART), M, W, 1e-5, grid))
    DX2, PART2 = torch.empty(M, W), torch.empty(1, 2, W)
    ref.ln_silu_bwd(X, w, b, G, DX2, PART2, 1e-5)
    _close(DX, DX2, 1e-4)
    _close(PART.sum(0), PART2[0], 1e-4)


@pytest.mark.parametrize("L", [1, 4, 6])
@pytest.mark.parametrize("bf16", [False, True])
def test_atomwise_gate_kernels(norm, L, bf16):
    torch.manual_seed(L)
    B, H = 6, 48
    dt = torch.bfloat16 if bf16 else torch.float32
    X = torch.randn(B, (L + 1) ** 2, H).to(dt)
    Gt = torch.randn(B, L * H)
    out, out2 = torch.empty_like(X), torch.empty_like(X)
    _ok(norm.emu_gate_l_fwd(L, _p(X), _p(Gt), _p(out), int(bf16), B, H))
    ref = CpuExtension()
    ref.gate_l_fwd(L, X, Gt, out2)
    _close(out, out2, 2 ** -7 if bf16 else 1e-5)
    DO = torch.randn_like(X.float()).to(dt)
    DX, DG = torch.empty_like(X), torch.empty(B, L * H)
    _ok(norm.emu_gate_l_bwd(L, _p(X), _p(Gt), _p(DO), _p(DX), _p(DG), int(bf16), B, H))
    DX2, DG2 = torch.empty_like(X), torch.empty(B, L * H)
    ref.gate_l_bwd(L, X, Gt, DO, DX2, DG2)
    _close(DX, DX2, 2 ** -7 if bf16 else 1e-5)
    _close(DG, DG2, 1e-4)
