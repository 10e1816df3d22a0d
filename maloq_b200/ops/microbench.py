"""Kernel micro-benchmarks (device-timed with CUDA events) for profiling single kernels.

    python -m maloq_b200.ops.microbench gemm [--bn 128] [--edges 43408]
    python -m maloq_b200.ops.microbench edge [--edges 43408]
    python -m maloq_b200.ops.microbench labels [--rows 236000] [--kind large]
    python -m maloq_b200.ops.microbench suite [--edges 43408] [--passes 2]

``gemm`` runs the first SO(2) convolution of one drug-like-config layer as one grouped
launch: M = edges, (N, K) = (1152, 1280), (1024, 1024), (768, 768), bf16 in/out.
``edge`` runs the fused gather/rotate/modulate kernel and its backward for the same layer.
Inputs exceed the 126 MB L2.  Prints time and achieved rate.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch


def _timeit(fn, iters=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(edges, bn):
    from . import kernels

    lib = kernels.lib()
    dev = torch.device("cuda", 0)
    shapes = [(1152, 1280), (1024, 1024), (768, 768)]
    A = torch.randn(edges, 19 * 256, device=dev).bfloat16()
    offs = [0, 1280, 1280 + 2048]
    As = [A[:, o:o + k] for o, (n, k) in zip(offs, shapes)]
    Ws = [torch.randn(n, k, device=dev).bfloat16() for n, k in shapes]
    Cs = [torch.empty(edges, n, device=dev, dtype=torch.bfloat16) for n, k in shapes]
    ms = _timeit(lambda: lib.gemm(As, Ws, Cs, [None] * 3, False, 0, 1.0, 1, bn))
    fl = sum(2 * edges * n * k for n, k in shapes)
    print(f"gemm bn={bn}: {ms * 1e3:.1f} us, {fl / ms / 1e9:.1f} TFLOP/s, error_status={kernels.error_status()}")


def bench_gemm_shape(M, N, K, bn, out_fp32=False):
    from . import kernels

    lib = kernels.lib()
    dev = torch.device("cuda", 0)
    A = torch.randn(M, K, device=dev).bfloat16()
    W = torch.randn(N, K, device=dev).bfloat16()
    C = torch.empty(M, N, device=dev, dtype=torch.float32 if out_fp32 else torch.bfloat16)
    ms = _timeit(lambda: lib.gemm([A], [W], [C], [None], False, 0, 1.0, 1, bn))
    print(f"gemm M={M} N={N} K={K} bn={bn}: {ms * 1e3:.1f} us, {2 * M * N * K / ms / 1e9:.1f} TFLOP/s")


def bench_edge(edges):
    from . import kernels

    lib = kernels.lib()
    dev = torch.device("cuda", 0)
    N = max(1, edges // 35)
    C, S, R, Cin = 128, 25, 19, 256
    x = torch.randn(N, S, C, device=dev)
    src = torch.randint(0, N, (edges,), device=dev)
    dst = torch.sort(torch.randint(0, N, (edges,), device=dev)).values
    rot = torch.randn(edges, R, S, device=dev)
    rad = torch.randn(edges, 12 * Cin, device=dev).bfloat16()
    A = torch.empty(edges, R * Cin, device=dev, dtype=torch.bfloat16)
    ms = _timeit(lambda: lib.gather_rotate_fwd(4, 2, x, None, src, dst, rot, rad, A, Cin, 0, None, None, 0))
    # node rows come from L2 (N*S*C*4 bytes once); per edge: rotation, radial row, A row
    byt = N * S * C * 4 + edges * (R * S * 4 + 12 * Cin * 2 + R * Cin * 2)
    print(f"gather_rotate_fwd: {ms * 1e3:.1f} us, {byt / ms / 1e9:.2f} TB/s algorithmic")
    dptr = torch.zeros(N + 1, dtype=torch.long, device=dev)
    dptr[1:] = torch.cumsum(torch.bincount(dst, minlength=N), 0)
    perm = torch.argsort(src, stable=True)
    sptr = torch.zeros(N + 1, dtype=torch.long, device=dev)
    sptr[1:] = torch.cumsum(torch.bincount(src, minlength=N), 0)
    DX = torch.empty(N, S, C, device=dev)
    DR = torch.empty_like(rad)
    ms = _timeit(lambda: lib.gather_rotate_bwd(4, 2, x, None, rot, rad, A, dptr, perm, sptr, DX, None, DR, Cin, 0,
                                               None, None, 0))
    Y2 = torch.randn(edges, R * C, device=dev).bfloat16()
    out_n = torch.empty(N, S, C, device=dev)
    out_e = torch.empty(edges, S, C, device=dev)
    gn = torch.randn(N, S, C, device=dev)
    dY = torch.empty(edges, R * C, device=dev, dtype=torch.bfloat16)
    for name, fn, byt2 in [
            ("rotate_back_scatter (node path)",
             lambda: lib.rotate_back_scatter(4, 2, Y2, 0, R, rot, dptr, None, out_n, 1.0),
             edges * (R * C * 2 + R * S * 4)),
            ("rotate_back_edge (edge path)", lambda: lib.rotate_back_edge(4, 2, Y2, 0, R, rot, out_e),
             edges * (R * C * 2 + R * S * 4 + S * C * 4)),
            ("rotate_grad (node path)", lambda: lib.rotate_grad(4, 2, gn, dst, rot, dY, None, R, 1.0),
             edges * (R * C * 2 + R * S * 4))]:
        t = _timeit(fn)
        print(f"{name}: {t * 1e3:.1f} us, {byt2 / t / 1e9:.2f} TB/s algorithmic")
    # per edge: rotation twice (both walks), radial row, dA row, radial gradient row
    byt = N * S * C * 4 * 2 + edges * (2 * R * S * 4 + 12 * Cin * 2 * 2 + R * Cin * 2)
    print(f"gather_rotate_bwd: {ms * 1e3:.1f} us, {byt / ms / 1e9:.2f} TB/s algorithmic, "
          f"error_status={kernels.error_status()}")


def bench_labels(rows, kind):
    """Fused block gather + coupled transform (``blocks_to_coupled``) and its inverse on ``rows``
    random atom pairs of the ``kind`` basis; bytes = block data + label rows (+ tables)."""
    from ..data import datasets
    from . import labels as lab

    dev = torch.device("cuda", 0)
    labeler = datasets.labeler_for(kind, dev)
    tbl = labeler.table
    g = torch.Generator().manual_seed(0)
    pt = torch.randint(0, tbl.n_types * tbl.n_types, (rows,), generator=g)
    na = torch.as_tensor(tbl.norb)[pt // tbl.n_types]
    nb = torch.as_tensor(tbl.norb)[pt % tbl.n_types]
    ptr = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(na * nb, 0)])
    n = int(ptr[-1])
    data = torch.randn(n, device=dev)
    ptr, pt = ptr.to(dev), pt.to(dev)
    D = labeler.target_len
    T = labeler.transform
    out = lab.blocks_to_coupled(data, ptr, pt, labeler.pos_t, T)
    ms1 = _timeit(lambda: lab.blocks_to_coupled(data, ptr, pt, labeler.pos_t, T))
    ms2 = _timeit(lambda: lab.coupled_to_blocks(out, ptr, pt, labeler.pos_t, T, n))
    byts = 4 * (n + rows * D)
    print(f"labels {kind} rows={rows} D={D}: blocks->coupled {ms1 * 1e3:.1f} us ({byts / ms1 / 1e6:.0f} GB/s), "
          f"coupled->blocks {ms2 * 1e3:.1f} us ({byts / ms2 / 1e6:.0f} GB/s)")


def suite_calls(edges=43408, device="cuda"):
    """One launch of every single-GPU kernel of the library at drug-like-config shapes (L=4,
    m=2, C=128, ``edges`` edges, 36 edges per node): a list of (name, zero-argument call that
    launches exactly one kernel).  Used to profile each kernel once (``suite``)."""
    from . import kernels
    from ..data import datasets
    from ..core.sph import J_matrices
    from ..models.so3 import CoefficientMapping
    from . import labels_native

    lib = kernels.lib()
    dev = torch.device(device, 0) if device == "cuda" else torch.device(device)
    torch.manual_seed(0)
    E, C, S, R, H, L, MM = edges, 128, 25, 19, 128, 4, 2
    Cin = 2 * C
    N = max(2, E // 36)
    x = torch.randn(N, S, C, device=dev)
    src = torch.randint(0, N, (E,), device=dev)
    dst = torch.sort(torch.randint(0, N, (E,), device=dev)).values
    dst_ptr = torch.zeros(N + 1, dtype=torch.long, device=dev)
    dst_ptr[1:] = torch.cumsum(torch.bincount(dst, minlength=N), 0)
    perm = torch.argsort(src, stable=True)
    sptr = torch.zeros(N + 1, dtype=torch.long, device=dev)
    sptr[1:] = torch.cumsum(torch.bincount(src, minlength=N), 0)
    vec = torch.randn(E, 3, device=dev)
    mapping = CoefficientMapping(L, MM)
    Js = J_matrices(L)
    flat = torch.cat([J.reshape(-1).float() for J in Js]).to(dev)
    joff = [sum((2 * k + 1) ** 2 for k in range(l)) for l in range(L + 1)]
    rot = torch.empty(E, R, S, device=dev)
    rad = torch.randn(E, 12 * Cin, device=dev).bfloat16()
    A = torch.empty(E, R * Cin, device=dev, dtype=torch.bfloat16)
    DR = torch.empty_like(rad)
    DX = torch.empty(N, S, C, device=dev)
    G = 4 * H  # gate scalars of the m = 0 block
    Y1 = torch.randn(E, G + R * H, device=dev).bfloat16()
    H1 = torch.empty(E, R * H, device=dev, dtype=torch.bfloat16)
    dY1 = torch.empty_like(Y1)
    Y2 = torch.randn(E, R * C, device=dev).bfloat16()
    out_n = torch.empty(N, S, C, device=dev)
    out_e = torch.empty(E, S, C, device=dev)
    g_n = torch.randn(N, S, C, device=dev)
    dY2 = torch.empty(E, R * C, device=dev, dtype=torch.bfloat16)
    shapes = [(1152, 1280), (1024, 1024), (768, 768)]
    Aop = torch.randn(E, 19 * 256, device=dev).bfloat16()
    offs = [0, 1280, 1280 + 2048]
    As = [Aop[:, o:o + k] for o, (n, k) in zip(offs, shapes)]
    Ws = [torch.randn(n, k, device=dev).bfloat16() for n, k in shapes]
    Cs = [torch.empty(E, n, device=dev, dtype=torch.bfloat16) for n, k in shapes]
    gy = torch.randn(E, 1152, device=dev).bfloat16()
    part = torch.empty(8, 1152, 1280, device=dev)
    wout = torch.empty(1152, 1280, device=dev)
    aw, ab = torch.rand(L + 1, C, device=dev), torch.rand(C, device=dev)
    ssum = torch.empty_like(x)
    rpart = torch.empty(148 * 4, L + 2, C, device=dev)
    xl = torch.randn(E, 128, device=dev)
    wl, bl = torch.rand(128, device=dev), torch.rand(128, device=dev)
    yl = torch.empty(E, 128, device=dev, dtype=torch.bfloat16)
    dxl = torch.empty_like(xl)
    lpart = torch.empty(148 * 4 * 8, 2, 128, device=dev)
    gates = torch.rand(N, L * C, device=dev)
    xg = torch.randn(N, S, C, device=dev)
    og, dxg, dg = torch.empty_like(xg), torch.empty_like(xg), torch.empty_like(gates)
    labeler = datasets.labeler_for("druglike", dev)
    D = labeler.target_len
    tbl = labeler.table
    pt = torch.randint(0, tbl.n_types * tbl.n_types, (E,), device=dev)
    sizes = torch.as_tensor(tbl.norb, device=dev)[pt // tbl.n_types] * torch.as_tensor(tbl.norb, device=dev)[
        pt % tbl.n_types]
    bptr = torch.zeros(E + 1, dtype=torch.long, device=dev)
    bptr[1:] = torch.cumsum(sizes, 0)
    data = torch.randn(int(bptr[-1]), device=dev)
    meta, coef = labels_native._tables(labeler.transform, True, dev, torch.float32)
    pos32 = labels_native._pos32(labeler.pos_t)
    coupled = torch.empty(E, D, device=dev)
    tgt = torch.randn(E, D, device=dev)
    mask = torch.as_tensor(tbl.mask, device=dev, dtype=torch.uint8).contiguous()
    lgrid = lib.fock_loss_grid(E * D)
    lstat = torch.empty(lgrid, 3, device=dev)
    lgrad = torch.empty_like(tgt)
    gstat = torch.tensor([1.0, 0.5], device=dev)
    ls, ms = mapping.l_harmonic.tolist(), mapping.m_complex.tolist()
    meta_h, coef_h = labels_native._tables(labeler.transform, False, dev, torch.float32)
    blocks_out = torch.empty_like(data)
    # device radius graph on a periodic Si/O cell of about E / 140 atoms (8 A cutoff)
    from ..data import structures
    from ..data.graph_gpu import grid_for

    st = structures.amorphous_sio2(np.random.default_rng(0), max(2000, E // 140))
    lo, ext, ncell, periodic = grid_for(st.pos, 8.0, st.cell)
    grid = [float(v) for v in lo] + [float(v) for v in ext] + [8.0]
    nc = [int(v) for v in ncell]
    pos_t = torch.as_tensor(st.pos, device=dev).contiguous()
    cell_id = torch.empty(len(st.z), dtype=torch.long, device=dev)
    lib.radius_graph_cells(pos_t, grid, nc, periodic, cell_id)
    order = torch.argsort(cell_id, stable=True)
    cstart = torch.zeros(nc[0] * nc[1] * nc[2] + 1, dtype=torch.long, device=dev)
    cstart[1:] = torch.cumsum(torch.bincount(cell_id, minlength=nc[0] * nc[1] * nc[2]), 0)
    tg = torch.arange(len(st.z), device=dev)
    cnt = torch.empty(len(st.z), dtype=torch.long, device=dev)
    lib.radius_graph_pass(pos_t, grid, nc, periodic, tg, order, cstart, cnt, None, None, None)
    gptr = torch.cumsum(cnt, 0) - cnt
    g_src = torch.empty(int(cnt.sum()), dtype=torch.long, device=dev)
    g_vec = torch.empty(int(cnt.sum()), 3, dtype=torch.float64, device=dev)
    return [
        ("edge_rotation", lambda: lib.edge_rotation(vec, flat, joff, L, ls, ms, rot)),
        ("gemm_tc2 (conv1 grouped, 2-SM)", lambda: lib.gemm(As, Ws, Cs, [None] * 3, False, 0, 1.0, 1, 128)),
        ("gemm_tc (weight grad, split-K)", lambda: lib.gemm([gy], [Aop[:, :1280]], [part], [None], True, 0, 1.0, 8,
                                                            128)),
        ("splitk_reduce", lambda: lib.splitk_reduce(part, wout, 0.0)),
        ("gather_rotate_fwd", lambda: lib.gather_rotate_fwd(L, MM, x, None, src, dst, rot, rad, A, Cin, 0, None, None,
                                                            0)),
        ("gather_rotate_bwd", lambda: lib.gather_rotate_bwd(L, MM, x, None, rot, rad, A, dst_ptr, perm, sptr, DX, None,
                                                            DR, Cin, 0, None, None, 0)),
        ("gate_fwd", lambda: lib.gate_fwd(L, MM, Y1, H1, H)),
        ("gate_bwd", lambda: lib.gate_bwd(L, MM, Y1, H1, dY1, H)),
        ("rotate_back_scatter", lambda: lib.rotate_back_scatter(L, MM, Y2, 0, R, rot, dst_ptr, None, out_n, 1.0)),
        ("rotate_back_edge", lambda: lib.rotate_back_edge(L, MM, Y2, 0, R, rot, out_e)),
        ("rotate_grad", lambda: lib.rotate_grad(L, MM, g_n, dst, rot, dY2, None, R, 1.0)),
        ("rms_norm_fwd", lambda: lib.rms_norm_fwd(L, x, x, aw, ab, out_n, ssum, 1e-5)),
        ("rms_norm_bwd", lambda: lib.rms_norm_bwd(L, ssum, g_n, g_n, aw, DX, rpart, 1e-5)),
        ("ln_silu_fwd", lambda: lib.ln_silu_fwd(xl, wl, bl, yl, 1e-5)),
        ("ln_silu_bwd", lambda: lib.ln_silu_bwd(xl, wl, bl, yl, dxl, lpart, 1e-5)),
        ("gate_l_fwd", lambda: lib.gate_l_fwd(L, xg, gates, og)),
        ("gate_l_bwd", lambda: lib.gate_l_bwd(L, xg, gates, og, dxg, dg)),
        ("basis_rows (blocks -> coupled)", lambda: lib.basis_rows(data, coupled, bptr, pt, pos32, meta, coef, D, E,
                                                                 True, False)),
        ("fock_loss_stats", lambda: lib.fock_loss_stats(coupled, tgt, pt, mask, lstat)),
        ("fock_loss_grad", lambda: lib.fock_loss_grad(coupled, tgt, pt, mask, gstat, lgrad)),
        ("basis_rows (coupled -> blocks)", lambda: lib.basis_rows(coupled, blocks_out, bptr, pt, pos32, meta_h,
                                                                 coef_h, D, E, False, True)),
        ("radius_graph cells", lambda: lib.radius_graph_cells(pos_t, grid, nc, periodic, cell_id)),
        ("radius_graph count", lambda: lib.radius_graph_pass(pos_t, grid, nc, periodic, tg, order, cstart, cnt,
                                                              None, None, None)),
        ("radius_graph fill", lambda: lib.radius_graph_pass(pos_t, grid, nc, periodic, tg, order, cstart, None,
                                                             gptr, g_src, g_vec)),
    ]


def bench_suite(edges, passes):
    """``passes`` passes over :func:`suite_calls` (one launch each), timing every kernel with
    CUDA events on the last pass."""
    from . import kernels

    calls = suite_calls(edges)
    print(f"suite: {len(calls)} kernels per pass, {passes} passes")
    for p in range(passes):
        for name, fn in calls:
            if p + 1 < passes:
                fn()
                continue
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            print(f"  {name:34s} {s.elapsed_time(e) * 1e3:9.1f} us")
    torch.cuda.synchronize()
    print(f"error_status={kernels.error_status()}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "edge", "shape", "labels", "suite"])
    ap.add_argument("--passes", type=int, default=2)
    ap.add_argument("--rows", type=int, default=236000)
    ap.add_argument("--kind", default="large")
    ap.add_argument("--M", type=int, default=32768)
    ap.add_argument("--N", type=int, default=1024)
    ap.add_argument("--K", type=int, default=1024)
    ap.add_argument("--fp32-out", action="store_true")
    ap.add_argument("--bn", type=int, default=128)
    ap.add_argument("--edges", type=int, default=43408)
    a = ap.parse_args(argv)
    if a.what == "shape":
        bench_gemm_shape(a.M, a.N, a.K, a.bn, a.fp32_out)
    elif a.what == "suite":
        bench_suite(a.edges, a.passes)
    elif a.what == "labels":
        bench_labels(a.rows, a.kind)
    elif a.what == "gemm":
        bench_gemm(a.edges, a.bn)
    else:
        bench_edge(a.edges)


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    main()
