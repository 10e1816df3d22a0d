"""Kernel micro-benchmarks (device-timed with CUDA events) for profiling single kernels.

    python -m maloq_b200.ops.microbench gemm [--bn 128] [--edges 43408]
    python -m maloq_b200.ops.microbench edge [--edges 43408]
    python -m maloq_b200.ops.microbench labels [--rows 236000] [--kind large]

``gemm`` runs the first SO(2) convolution of one drug-like-config layer as one grouped
launch: M = edges, (N, K) = (1152, 1280), (1024, 1024), (768, 768), bf16 in/out.
``edge`` runs the fused gather/rotate/modulate kernel and its backward for the same layer.
Inputs exceed the 126 MB L2.  Prints time and achieved rate.
"""

from __future__ import annotations

import argparse
import os
import sys

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
    rad = torch.randn(edges, 12 * Cin, device=dev)
    A = torch.empty(edges, R * Cin, device=dev, dtype=torch.bfloat16)
    ms = _timeit(lambda: lib.gather_rotate_fwd(4, 2, x, None, src, dst, rot, rad, A, Cin))
    byt = edges * (S * Cin * 4 + R * S * 4 + 12 * Cin * 4 + R * Cin * 2)
    print(f"gather_rotate_fwd: {ms * 1e3:.1f} us, {byt / ms / 1e9:.2f} TB/s algorithmic")
    DS = torch.empty(edges, S, C, device=dev)
    DD = torch.empty(edges, S, C, device=dev)
    DR = torch.empty_like(rad)
    ms = _timeit(lambda: lib.gather_rotate_bwd(4, 2, x, None, src, dst, rot, rad, A, DS, DD, None, DR, Cin))
    byt = edges * (S * Cin * 4 * 2 + R * S * 4 + 12 * Cin * 4 * 2 + R * Cin * 2)
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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "edge", "shape", "labels"])
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
    elif a.what == "labels":
        bench_labels(a.rows, a.kind)
    elif a.what == "gemm":
        bench_gemm(a.edges, a.bn)
    else:
        bench_edge(a.edges)


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    main()
