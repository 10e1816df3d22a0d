"""Whole ops and a model training step on the CUDA kernel sources, run on the CPU emulator
(``tests/emulated_extension.py``): the label conversions and basis transform (``labels.cu``), the
device radius graph (``graph.cu``), the edge rotation and fused loss (``misc.cu``) and the
model's kernel path (edge frame, norms, gates, head gate) against the PyTorch definitions.  The
kernels are built with the index checks on (``MALOQ_BOUNDS_CHECK``); every test also asserts
that no kernel recorded an error code."""
import numpy as np
import pytest
import torch

from tests.emulated_extension import load_libraries, use_emulated_extension


@pytest.fixture(scope="module")
def libs(tmp_path_factory):
    libs = load_libraries(tmp_path_factory.mktemp("emu_ops"), defines=("MALOQ_BOUNDS_CHECK=1",))
    if libs is None:
        pytest.skip("needs g++ and the CUDA headers")
    return libs


def _labels_case(kind, n_mol, dtype, seed=0):
    from maloq_b200.data import datasets

    labeler = datasets.labeler_for(kind, "cpu")
    samples = datasets.build_samples(kind, n_mol, seed=seed)
    tbl = labeler.table
    ptrs, pts, n = [0], [], 0
    for s in samples:
        rows, cols = labeler.pairs(s)
        nz = tbl.norb[tbl.z_to_type[s.z]]
        for sz in nz[rows] * nz[cols]:
            n += int(sz)
            ptrs.append(n)
        pts.append(tbl.pair_type(s.z[rows], s.z[cols]))
    g = torch.Generator().manual_seed(seed)
    data = torch.randn(n, generator=g, dtype=torch.float64).to(dtype)
    return labeler, data, torch.tensor(ptrs), torch.as_tensor(np.concatenate(pts), dtype=torch.long), n


@pytest.mark.parametrize("kind,n_mol,dtype", [("druglike", 1, torch.float32), ("druglike", 1, torch.float64),
                                              ("large", 1, torch.float32)])
def test_label_ops_on_emulated_kernels(monkeypatch, libs, kind, n_mol, dtype):
    from maloq_b200.ops import basis_transform as bt
    from maloq_b200.ops import labels as lab

    labeler, data, ptr, pt, n = _labels_case(kind, n_mol, dtype)
    pos, T = labeler.pos_t.cpu(), labeler.transform
    ref_lab = lab._ref_m2l(data, ptr, pt, pos)
    ref_c = ref_lab.double() @ T.W_global_inv.double()
    x = ref_c.to(dtype)
    ref_h = x.double() @ T.W_global.double()
    ref_d = lab._ref_l2m(ref_h, ptr, pt, pos, n)
    ext = use_emulated_extension(monkeypatch, libs)
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    got_lab = lab.matrix_to_labels(data, ptr, pt, pos)
    assert torch.equal(got_lab, ref_lab)
    assert torch.equal(lab.labels_to_matrix(got_lab, ptr, pt, pos, n), lab._ref_l2m(ref_lab, ptr, pt, pos, n))
    for got, ref in ((lab.blocks_to_coupled(data, ptr, pt, pos, T), ref_c),
                     (bt.apply_transform(x, T, inverse=False), ref_h),
                     (lab.coupled_to_blocks(x, ptr, pt, pos, T, n), ref_d)):
        got = got.double()
        assert (got - ref).abs().max() <= tol * max(1.0, ref.abs().max().item())
    assert ext.emulated_calls["basis_rows"] == 5
    assert ext.emulated_error_word() == 0


def test_label_gather_with_a_bad_pair_type_records_an_error(monkeypatch, libs):
    """A pair type outside the position table skips the access and records the bounds code."""
    from maloq_b200.ops import labels as lab

    labeler, data, ptr, pt, n = _labels_case("druglike", 1, torch.float32)
    pt = pt.clone()
    pt[0] = labeler.pos_t.shape[0] + 3
    ext = use_emulated_extension(monkeypatch, libs)
    out = lab.matrix_to_labels(data, ptr, pt, labeler.pos_t.cpu())
    assert ext.emulated_error_word() == 5  # ERR_BOUNDS
    assert torch.all(out[0] == 0)


@pytest.mark.parametrize("periodic", [False, True])
@pytest.mark.parametrize("subset", [False, True])
def test_device_radius_graph_on_emulated_kernels(monkeypatch, libs, periodic, subset):
    from maloq_b200.data.graph import radius_graph
    from maloq_b200.data.graph_gpu import radius_graph_device

    rng = np.random.default_rng(3)
    cell = np.array([11.0, 12.5, 10.5]) if periodic else None
    pos = rng.uniform(0, 10.5, (150, 3))
    cutoff = 3.2
    src, dst, vec = radius_graph(pos, cutoff, cell)
    targets = np.arange(0, 150, 3) if subset else None
    ext = use_emulated_extension(monkeypatch, libs)
    s, d, v, ptr = radius_graph_device(pos, cutoff, cell, targets=targets, device="cpu")
    assert ext.emulated_calls == {"radius_graph_cells": 1, "radius_graph_pass": 2}
    if subset:  # the host graph restricted to the target rows, dst renumbered
        keep = np.isin(dst, targets)
        src, dst, vec = src[keep], np.searchsorted(targets, dst[keep]), vec[keep]
    assert np.array_equal(s.numpy(), src) and np.array_equal(d.numpy(), dst)
    assert np.allclose(v.numpy(), vec, atol=1e-12)
    assert ptr[-1].item() == len(src)
    assert ext.emulated_error_word() == 0


@pytest.mark.parametrize("lmax,mmax", [(2, 2), (4, 2), (6, 2), (6, 6)])
def test_edge_rotation_kernel_matches_wigner_matrices(libs, lmax, mmax):
    """The kernel's rows of D(0, -beta, -alpha) against the stand-in's fp64 Wigner matrices, for
    random directions and the poles (beta = 0 and pi), over a strided vector view."""
    from maloq_b200.core import sph
    from maloq_b200.models.so3 import CoefficientMapping
    from tests.cpu_extension import CpuExtension
    from tests.emulated_extension import EmulatedExtension

    Js = sph.J_matrices(lmax)
    flat = torch.cat([J.reshape(-1).float() for J in Js]).contiguous()
    joff = [sum((2 * q + 1) ** 2 for q in range(l)) for l in range(lmax + 1)]
    mp = CoefficientMapping(lmax, mmax)
    ls, ms = mp.l_harmonic.tolist(), mp.m_complex.tolist()
    g = torch.Generator().manual_seed(lmax + mmax)
    attr = torch.randn(40, 4, generator=g)
    attr[0, 1:] = torch.tensor([0.3, 0.0, 0.0])  # along +y in the model frame (the polar axis)
    attr[1, 1:] = torch.tensor([-2.0, 0.0, 0.0])
    vec = attr[:, 1:]  # strided view: leading dimension 4
    R, S = len(ls), (lmax + 1) ** 2
    got, ref = torch.empty(40, R, S), torch.empty(40, R, S)
    emu = EmulatedExtension(libs)
    emu.edge_rotation(vec, flat, joff, lmax, ls, ms, got)
    CpuExtension().edge_rotation(vec.contiguous(), flat, joff, lmax, ls, ms, ref)
    assert (got - ref).abs().max() < 2e-5
    assert emu.emulated_error_word() == 0


@pytest.mark.parametrize("extra", [{}, dict(edge_chunk=40)])
def test_model_training_step_on_emulated_kernels(monkeypatch, libs, extra):
    """Forward, loss and every parameter gradient of a two-layer Fock model with every plain
    kernel of the step (edge frame, norms, gates, head gate, rotation, radial inputs, loss) run
    from its CUDA source on the emulator (GEMMs from the stand-in), against the PyTorch path."""
    from tests.test_kernel_path_cpu import _model, _step

    bb, hd, b, lab = _model(2, "source-target", **extra)
    ref = _step(bb, hd, b, lab)
    ext = use_emulated_extension(monkeypatch, libs)
    got = _step(bb, hd, b, lab)
    expected = {"edge_rotation", "gather_rotate_fwd", "gather_rotate_bwd", "gate_fwd", "gate_bwd",
                "rotate_back_scatter", "rotate_back_edge", "rotate_grad", "rms_norm_fwd", "rms_norm_bwd",
                "ln_silu_fwd", "ln_silu_bwd", "gate_l_fwd", "gate_l_bwd", "head_gate_fwd", "head_gate_bwd",
                "fock_loss_stats", "fock_loss_grad"}
    assert expected <= set(ext.emulated_calls), expected - set(ext.emulated_calls)
    for a, r in zip(got[:3], ref[:3]):
        assert abs(a - r) <= 3e-2 * abs(r), (a, r)
    assert set(got[3]) == set(ref[3])
    worst = max((float((got[3][n] - g).norm() / (g.norm() + 1e-12)), n) for n, g in ref[3].items())
    assert worst[0] < 5e-2, worst
    assert ext.emulated_error_word() == 0


@pytest.mark.parametrize("M,N,dtype,col0", [(0, 5, torch.float32, 0), (1, 3, torch.bfloat16, 0),
                                            (300, 40, torch.bfloat16, 8), (4096, 7, torch.float32, 2),
                                            (9000, 70, torch.bfloat16, 16), (20000, 33, torch.float32, 1)])
def test_colsum_kernel(libs, M, N, dtype, col0):
    """Fixed-order column sums of a row-strided slice (one stage for short matrices, row chunks
    plus a second pass for long ones) against an fp64 sum, twice with the same bits."""
    from tests.emulated_extension import EmulatedExtension

    ext = EmulatedExtension(libs)
    g = torch.Generator().manual_seed(M + N)
    full = torch.randn(M, N + col0 + 5, generator=g).to(dtype)
    X = full[:, col0:col0 + N]
    out = torch.full((N,), float("nan"))
    ext.colsum(X, out)
    ref = X.double().sum(0)
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-4 * max(1.0, M ** 0.5))
    again = torch.empty(N)
    ext.colsum(X, again)
    assert torch.equal(out, again)
    assert ext.emulated_error_word() == 0


def test_colsum_chunk_count(libs):
    """The chunk count and the launch's chunks: rows that do not split evenly leave trailing
    chunks empty, which the launcher does not launch or read back."""
    m = libs["misc"]
    assert m.emu_colsum_chunks(4096, 128) == 1
    assert m.emu_colsum_chunks(45948, 128) == 148  # four 32-column blocks, ~592 CTAs
    assert m.emu_colsum_chunks(151553, 8) == 592
    for M, N in ((151553, 8), (45948, 128), (5000, 3072)):
        P = m.emu_colsum_chunks(M, N)
        chunk = -(-M // P)
        used = -(-M // chunk)
        assert 1 <= used <= P and (used - 1) * chunk < M <= used * chunk


def test_weight_pack_kernel(libs):
    """The weight operand copies (bf16 cast, transpose of a matrix and of a batch of matrices,
    SO(2) pair matrix and its transpose) and the pair-matrix gradient, in one call of more jobs
    than one launch takes, against their PyTorch definitions."""
    from maloq_b200.ops import weights as W
    from tests.emulated_extension import EmulatedExtension

    ext = EmulatedExtension(libs)
    g = torch.Generator().manual_seed(3)
    srcs, dsts, kinds, refs = [], [], [], []
    for i in range(60):  # > 48 jobs: two launches
        kind = i % 5
        h, k = 1 + i % 7, 1 + (3 * i) % 11
        if kind == 1 and i % 2:
            S = torch.randn(3, 2 * h, k, generator=g)
        elif kind == 4:
            S = torch.randn(2 * h, 2 * k, generator=g)
        else:
            S = torch.randn(2 * h, k, generator=g)
        ref = [lambda: S, lambda: S.transpose(-1, -2), lambda: W._pair(S), lambda: W._pair(S).t(),
               lambda: W.pair_grad(S)][kind]()
        refs.append(ref if kind == 4 else ref.to(torch.bfloat16))
        dsts.append(torch.full(ref.shape, float("nan"), dtype=torch.float32 if kind == 4 else torch.bfloat16))
        srcs.append(S)
        kinds.append(kind)
    ext.weight_pack(srcs, dsts, kinds)
    for d, r, kd in zip(dsts, refs, kinds):
        if kd == 4:
            assert torch.allclose(d, r, rtol=1e-6, atol=1e-6)
        else:
            assert torch.equal(d, r), kd
    assert ext.emulated_error_word() == 0


def test_colsum_segments_kernel(libs):
    """Row-segment sums (an empty segment included) against fp64 sums."""
    from tests.emulated_extension import EmulatedExtension

    ext = EmulatedExtension(libs)
    g = torch.Generator().manual_seed(5)
    X = torch.randn(140, 75, generator=g)
    seg = [0, 3, 3, 40, 100, 140]
    out = torch.full((len(seg) - 1, 75), float("nan"))
    ext.colsum_segments(X, seg, out)
    ref = torch.stack([X[a:b].double().sum(0) for a, b in zip(seg[:-1], seg[1:])])
    assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-4)
    assert ext.emulated_error_word() == 0


def test_weight_cache_refreshed_in_place_by_weight_pack(monkeypatch, libs):
    """On the kernel path the bf16 weight copies come from the weight-pack kernel; after an
    optimizer step the hook rewrites every live copy in place (same tensors, new values) in one
    launch, and the pair-matrix gradients of several weights come from one call."""
    from maloq_b200.ops import weights as W

    ext = use_emulated_extension(monkeypatch, libs)
    W.invalidate()
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(8, 6))
    q = torch.nn.Parameter(torch.randn(3, 4, 5))
    opt = torch.optim.SGD([p, q], lr=0.1)
    first = None
    for step in range(3):
        wr, wi = p.detach()[:4], p.detach()[4:]
        pair = torch.cat([torch.cat([wr, -wi], 1), torch.cat([wi, wr], 1)], 0)
        got = [W.pair_bf16(p), W.pair_bf16_t(p), W.bf16(p), W.bf16_t(q)]
        for a, b in zip(got, [pair, pair.t(), p.detach(), q.detach().transpose(-1, -2)]):
            assert torch.equal(a, b.bfloat16())
        if first is None:
            first = got
        else:  # the same tensors, rewritten by the hook
            assert all(a is b for a, b in zip(got, first))
        (p.sum() + (q * step).sum()).backward()
        before = ext.emulated_calls.get("weight_pack", 0)
        opt.step()
        assert ext.emulated_calls["weight_pack"] == before + 1
        opt.zero_grad()
    dPs = [torch.randn(8, 12), torch.randn(4, 2)]
    before = ext.emulated_calls["weight_pack"]
    for g, d in zip(W.pair_grads(dPs), dPs):
        assert torch.allclose(g, W.pair_grad(d))
    assert ext.emulated_calls["weight_pack"] == before + 1
    assert ext.emulated_error_word() == 0
    W.invalidate()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gate_with_silu_gates_kernel(libs, dtype):
    """The l-outer gate fed the gate pre-activations (SiLU inside the kernels) against
    ``gate(silu(pre), x)`` in PyTorch, forward and both gradients."""
    from maloq_b200.ops import reference as R
    from tests.emulated_extension import EmulatedExtension

    ext = EmulatedExtension(libs)
    L, B, H = 4, 13, 24
    g = torch.Generator().manual_seed(2)
    x = torch.randn(B, (L + 1) ** 2, H, generator=g).to(dtype)
    pre = torch.randn(B, L * H, generator=g) * 2
    dout = torch.randn(B, (L + 1) ** 2, H, generator=g).to(dtype)
    idx = torch.tensor([l - 1 for l in range(1, L + 1) for _ in range(2 * l + 1)])
    xr, pr = x.float().requires_grad_(), pre.clone().requires_grad_()
    ref = R.gate(torch.nn.functional.silu(pr), xr, idx, L)
    ref.backward(dout.float())
    out = torch.empty_like(x)
    ext.gate_l_fwd(L, x, pre, out, True)
    dx, dpre = torch.empty_like(x), torch.empty_like(pre)
    ext.gate_l_bwd(L, x, pre, dout, dx, dpre, True)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert torch.allclose(out.float(), ref.detach(), rtol=tol, atol=tol)
    assert torch.allclose(dx.float(), xr.grad, rtol=tol, atol=tol)
    assert torch.allclose(dpre, pr.grad, rtol=1e-4 if dtype == torch.float32 else 2e-2, atol=1e-4 if dtype == torch.float32 else 2e-2)
    assert ext.emulated_error_word() == 0
