"""The extension's bindings backed by the CUDA kernel sources run on the CPU emulator.

``EmulatedExtension`` subclasses the PyTorch stand-in (``tests/cpu_extension.py``): every binding
whose kernel is a plain CUDA kernel (edge frame, norms and gates, edge rotation, Fock loss,
radial inputs, label rows, radius graph) calls the unmodified kernel source from ``ops/csrc``,
compiled for the host by ``tests/kernel_emu_build.py`` and launched through its own host
launcher on ``tests/csrc/host_emu.cuh`` (one host thread per CUDA thread, real block barriers,
warp shuffles, alignment-checked vector loads).  The argument mapping of each method is the one
of the binding in ``ops/csrc/bindings.cpp``.  GEMMs (tensor-core kernels) and the peer-memory
kernels stay with the stand-in.

With ``use_emulated_extension(monkeypatch, folder)`` the op layer runs its kernel path on CPU
tensors through these kernels, so whole ops (label conversion, device radius graph, loss, a
model step) exercise the kernels' real index arithmetic, shared-memory use and reductions.
"""

from __future__ import annotations

import ctypes

import torch

from tests.cpu_extension import CpuExtension, _Recorder
from tests.kernel_emu_build import build

P, I, LL, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float

SIGNATURES = {
    "edge": {
        "emu_gather_rotate_fwd": [I, I, P, P, P, P, P, P, P, I, I, I, LL],
        "emu_gather_rotate_bwd": [I, I, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I],
        "emu_rotate_back_scatter": [I, I, P, I, I, P, P, P, P, I, I, I, F],
        "emu_rotate_back_edge": [I, I, P, I, I, P, P, I, I, I],
        "emu_rotate_grad": [I, I, P, P, P, P, P, I, I, I, F],
        "emu_gate_fwd": [I, I, P, P, I, I],
        "emu_gate_bwd": [I, I, P, P, P, I, I],
        "emu_node_reduce": [P, P, P, P, P, P, I, I, LL, LL],
    },
    "norm": {
        "emu_norm_grid": [LL],
        "emu_rms_norm_fwd": [I, P, P, P, P, P, I, P, I, I, F],
        "emu_rms_norm_bwd": [I, P, P, I, P, P, P, P, I, I, F, I],
        "emu_ln_silu_fwd": [P, P, P, P, I, I, F],
        "emu_ln_silu_bwd": [P, P, P, P, P, P, I, I, F, I],
        "emu_gate_l_fwd": [I, P, P, P, I, I, I],
        "emu_gate_l_bwd": [I, P, P, P, P, P, I, I, I],
        "emu_gate_l_fwd_s": [I, P, P, P, I, I, I, I],
        "emu_gate_l_bwd_s": [I, P, P, P, P, P, I, I, I, I],
        "emu_head_gate_fwd": [I, P, P, P, I, F, I, I, I],
        "emu_head_gate_bwd": [I, P, P, P, P, P, I, F, I, I, I],
    },
    "misc": {
        "emu_edge_rotation": [P, LL, P, P, I, P, P, I, P, I],
        "emu_fock_loss_grid": [LL],
        "emu_fock_loss_stats": [P, P, P, P, I, LL, P, I, LL],
        "emu_colsum_chunks": [LL, I],
        "emu_colsum": [P, I, LL, I, LL, P, I, P],
        "emu_weight_pack": [I, P, P, P, P, P, P],
        "emu_colsum_segments": [P, I, LL, P, I, P],
        "emu_fock_loss_grad": [P, P, P, P, I, LL, P, P, LL],
        "emu_edge_inputs": [P, P, P, LL, P, P, LL, P, F, P, LL, I, I],
    },
    "labels": {
        "emu_basis_rows": [P, LL, P, LL, P, P, P, I, P, P, I, I, LL, LL, LL, I, I, I],
    },
    "graph": {
        "emu_radius_graph_cells": [P, LL, P, P, P, P],
        "emu_radius_graph_pass": [P, P, P, P, P, I, P, P, P, P, P, P, I],
    },
}
_INT_RESULT = {"emu_norm_grid", "emu_fock_loss_grid", "emu_colsum_chunks"}


def load_libraries(folder, names=tuple(SIGNATURES), defines=()):
    """Build and load the emulated kernel libraries; None when the host toolchain is missing."""
    libs = {}
    for name in names:
        lib = build(name, str(folder), defines=defines)
        if lib is None:
            return None
        for fn, args in SIGNATURES[name].items():
            f = getattr(lib, fn)
            f.argtypes = args
            f.restype = ctypes.c_int if fn in _INT_RESULT else ctypes.c_char_p
        lib.emu_error_word.restype = ctypes.c_int
        libs[name] = lib
    return libs


def _p(t):
    return None if t is None else t.data_ptr()


def _check(r):
    if r is not None:
        raise RuntimeError(f"maloq_b200 kernel: {r.decode()}")


def _i32(v):
    return (ctypes.c_int * len(v))(*[int(x) for x in v])


class EmulatedExtension(CpuExtension):
    """The stand-in with the plain CUDA kernels replaced by their emulated sources."""

    def __init__(self, libs, barrier_timeout=30.0):
        super().__init__(barrier_timeout)
        self.e, self.n = libs["edge"], libs["norm"]
        self.m, self.lb, self.g = libs["misc"], libs["labels"], libs["graph"]
        self.emulated_calls = {}

    def _count(self, name):
        self.emulated_calls[name] = self.emulated_calls.get(name, 0) + 1

    def emulated_error_word(self):
        """The first error code any emulated kernel recorded since the last call (then cleared)."""
        codes = [lib.emu_error_word() for lib in (self.e, self.n, self.m, self.lb, self.g)]
        return next((c for c in codes if c), 0)

    # ---------------------------------------------------------------- edge frame
    def gather_rotate_fwd(self, L, MM, X, XE, src, dst, rot, rad, A, Cin, peers, halo_owner, halo_row, n_own):
        if peers:
            return super().gather_rotate_fwd(L, MM, X, XE, src, dst, rot, rad, A, Cin, peers, halo_owner, halo_row,
                                             n_own)
        assert A.numel() == src.numel() * rot.shape[1] * Cin
        self._count("gather_rotate_fwd")
        _check(self.e.emu_gather_rotate_fwd(L, MM, _p(X), _p(XE), _p(src), _p(dst), _p(rot), _p(rad), _p(A),
                                            src.shape[0], X.shape[2], Cin, X.shape[0]))

    def gather_rotate_bwd(self, L, MM, X, XE, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DXE, DRAD, Cin,
                          peers=0, halo_owner=None, halo_row=None, n_own=0, recv=0, recv_slot=None):
        if peers:
            return super().gather_rotate_bwd(L, MM, X, XE, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DXE, DRAD,
                                             Cin, peers, halo_owner, halo_row, n_own, recv, recv_slot)
        N = DX.shape[0]
        assert dst_ptr.numel() == N + 1 and src_ptr.numel() == N + 1
        self._count("gather_rotate_bwd")
        _check(self.e.emu_gather_rotate_bwd(L, MM, _p(X), _p(XE), _p(rot), _p(rad), _p(dA), _p(dst_ptr),
                                            _p(src_perm), _p(src_ptr), _p(DX), _p(DXE), _p(DRAD), N, rot.shape[0],
                                            X.shape[2], Cin))

    def rotate_back_scatter(self, L, MM, Y, koff, Rk, rot, dst_ptr, base, out, scale):
        self._count("rotate_back_scatter")
        _check(self.e.emu_rotate_back_scatter(L, MM, _p(Y), Y.shape[1], koff, _p(rot), _p(dst_ptr), _p(base),
                                              _p(out), out.shape[0], out.shape[2], Rk, scale))

    def rotate_back_edge(self, L, MM, Y, koff, Rk, rot, out):
        self._count("rotate_back_edge")
        _check(self.e.emu_rotate_back_edge(L, MM, _p(Y), Y.shape[1], koff, _p(rot), _p(out), out.shape[0],
                                           out.shape[2], Rk))

    def rotate_grad(self, L, MM, G, rows, rot, DY, DYf, Rk, scale):
        self._count("rotate_grad")
        _check(self.e.emu_rotate_grad(L, MM, _p(G), _p(rows), _p(rot), _p(DY), _p(DYf), rot.shape[0], G.shape[2],
                                      Rk, scale))

    def gate_fwd(self, L, MM, Y1, H1, H):
        self._count("gate_fwd")
        _check(self.e.emu_gate_fwd(L, MM, _p(Y1), _p(H1), Y1.shape[0], H))

    def gate_bwd(self, L, MM, Y1, dH1, dY1, H):
        self._count("gate_bwd")
        _check(self.e.emu_gate_bwd(L, MM, _p(Y1), _p(dH1), _p(dY1), Y1.shape[0], H))

    def node_reduce(self, DDST, dst_ptr, DSRC, src_perm, src_ptr, DX):
        self._count("node_reduce")
        N = DX.shape[0]
        SC = DX.numel() // max(1, N)
        _check(self.e.emu_node_reduce(_p(DDST), _p(dst_ptr), _p(DSRC), _p(src_perm), _p(src_ptr), _p(DX), N, SC,
                                      0 if DDST is None else DDST.shape[0], 0 if DSRC is None else DSRC.shape[0]))

    # ---------------------------------------------------------------- norms and gates
    def norm_grid(self, rows):
        return self.n.emu_norm_grid(rows)

    def rms_norm_fwd(self, L, X, RES, aw, ab, OUT, SUM, eps):
        self._count("rms_norm_fwd")
        _check(self.n.emu_rms_norm_fwd(L, _p(X), _p(RES), _p(aw), _p(ab), _p(OUT), int(OUT.dtype == torch.bfloat16),
                                       _p(SUM), X.shape[0], X.shape[2], eps))

    def rms_norm_bwd(self, L, Sx, G, GS, aw, DX, PART, eps):
        self._count("rms_norm_bwd")
        _check(self.n.emu_rms_norm_bwd(L, _p(Sx), _p(G), int(G.dtype == torch.bfloat16), _p(GS), _p(aw), _p(DX),
                                       _p(PART), Sx.shape[0], Sx.shape[2], eps, PART.shape[0]))

    def ln_silu_fwd(self, X, w, b, OUT, eps):
        self._count("ln_silu_fwd")
        _check(self.n.emu_ln_silu_fwd(_p(X), _p(w), _p(b), _p(OUT), X.shape[0], X.shape[1], eps))

    def ln_silu_bwd(self, X, w, b, G, DX, PART, eps):
        self._count("ln_silu_bwd")
        _check(self.n.emu_ln_silu_bwd(_p(X), _p(w), _p(b), _p(G), _p(DX), _p(PART), X.shape[0], X.shape[1], eps,
                                      PART.shape[0] // 8))

    def gate_l_fwd(self, L, X, Gt, OUT, silu_gates=False):
        self._count("gate_l_fwd")
        _check(self.n.emu_gate_l_fwd_s(L, _p(X), _p(Gt), _p(OUT), int(X.dtype == torch.bfloat16), X.shape[0],
                                       X.shape[2], int(silu_gates)))

    def gate_l_bwd(self, L, X, Gt, DO, DX, DG, silu_gates=False):
        self._count("gate_l_bwd")
        _check(self.n.emu_gate_l_bwd_s(L, _p(X), _p(Gt), _p(DO), _p(DX), _p(DG), int(X.dtype == torch.bfloat16),
                                       X.shape[0], X.shape[2], int(silu_gates)))

    def head_gate_fwd(self, L, X, SV, A, act, scale, absg):
        assert A.shape == X.shape and SV.shape == (X.shape[0], (L + 1) * X.shape[2])
        self._count("head_gate_fwd")
        _check(self.n.emu_head_gate_fwd(L, _p(X), _p(SV), _p(A), act, scale, int(absg), X.shape[0], X.shape[2]))

    def head_gate_bwd(self, L, X, SV, DA, DX, DSV, act, scale, absg):
        self._count("head_gate_bwd")
        _check(self.n.emu_head_gate_bwd(L, _p(X), _p(SV), _p(DA), _p(DX), _p(DSV), act, scale, int(absg), X.shape[0],
                                        X.shape[2]))

    # ---------------------------------------------------------------- rotation, inputs, loss
    def edge_rotation(self, vec, J, joff, L, row_l, row_m, ROT):
        assert vec.dtype == torch.float32 and vec.stride(1) == 1
        jo = list(joff) + [0] * (7 - len(joff))
        self._count("edge_rotation")
        _check(self.m.emu_edge_rotation(_p(vec), vec.stride(0), _p(J), _i32(jo), L, _i32(row_l), _i32(row_m),
                                        len(row_l), _p(ROT), vec.shape[0]))

    def edge_inputs(self, src_z, dst_z, edge_attr, src_table, dst_table, offset, coeff, OUT):
        E, C, NB = src_z.numel(), src_table.shape[1], offset.numel()
        assert OUT.dtype == torch.bfloat16 and tuple(OUT.shape) == (E, 2 * C + NB)
        assert edge_attr.is_contiguous() and edge_attr.shape[0] == E
        self._count("edge_inputs")
        _check(self.m.emu_edge_inputs(_p(src_z), _p(dst_z), _p(edge_attr), edge_attr.shape[1], _p(src_table),
                                      _p(dst_table), src_table.shape[0], _p(offset), coeff, _p(OUT), E, C, NB))

    def colsum(self, X, out):
        assert X.dim() == 2 and X.dtype in (torch.float32, torch.bfloat16) and out.dtype == torch.float32
        assert (X.shape[1] <= 1 or X.stride(1) == 1) and out.is_contiguous() and out.numel() == X.shape[1]
        self._count("colsum")
        M, N = X.shape
        P = self.m.emu_colsum_chunks(M, N)
        part = torch.empty(P, N, dtype=torch.float32) if P > 1 else None
        _check(self.m.emu_colsum(_p(X), int(X.dtype == torch.bfloat16), M, N, X.stride(0) if M > 1 else N,
                                 _p(part), P, _p(out)))

    def colsum_segments(self, X, seg, out):
        assert X.dim() == 2 and X.dtype == torch.float32 and (X.shape[1] <= 1 or X.stride(1) == 1)
        assert out.is_contiguous() and out.numel() == (len(seg) - 1) * X.shape[1]
        self._count("colsum_segments")
        s = (ctypes.c_longlong * len(seg))(*[int(v) for v in seg])
        _check(self.m.emu_colsum_segments(_p(X), X.shape[1], X.stride(0) if X.shape[0] > 1 else X.shape[1], s,
                                          len(seg) - 1, _p(out)))

    def weight_pack(self, srcs, dsts, kinds):
        n = len(srcs)
        shp = [(S.shape[0] if S.dim() == 3 else 1, S.shape[-2] if S.dim() >= 2 else 1, S.shape[-1]) for S in srcs]
        for S, D in zip(srcs, dsts):
            assert S.dtype == torch.float32 and S.is_contiguous() and D.is_contiguous()
        self._count("weight_pack")
        ptrs = lambda ts: (ctypes.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
        _check(self.m.emu_weight_pack(n, ptrs(srcs), ptrs(dsts), _i32([b for b, _, _ in shp]),
                                      _i32([r for _, r, _ in shp]), _i32([c for _, _, c in shp]), _i32(kinds)))

    def fock_loss_grid(self, n):
        return self.m.emu_fock_loss_grid(n)

    def fock_loss_stats(self, O, T, pt, mask, part):
        assert mask.dtype == torch.uint8 and O.is_contiguous() and T.is_contiguous()
        self._count("fock_loss_stats")
        _check(self.m.emu_fock_loss_stats(_p(O), _p(T), _p(pt), _p(mask), O.shape[1], O.shape[0], _p(part),
                                          part.shape[0], mask.shape[0]))

    def fock_loss_grad(self, O, T, pt, mask, gstat, G):
        assert gstat.dtype == torch.float32 and gstat.numel() >= 2 and gstat.stride(0) == 1
        self._count("fock_loss_grad")
        _check(self.m.emu_fock_loss_grad(_p(O), _p(T), _p(pt), _p(mask), O.shape[1], O.shape[0], _p(gstat), _p(G),
                                         mask.shape[0]))

    # ---------------------------------------------------------------- label rows
    def basis_rows(self, inp, out, ptr, pt, pos, meta, coef, d_in, rows, gather, scatter):
        assert inp.dtype == out.dtype == coef.dtype and inp.dtype in (torch.float32, torch.float64)
        assert meta.dtype == torch.int32 and meta.shape[1] == 4 and meta.is_contiguous()
        d_out = meta.shape[0]
        d_pos, n_pt, n_data = 0, 0, 0
        if gather or scatter:
            assert pos.dtype == torch.int32 and ptr.numel() >= rows and pt.numel() >= rows
            d_pos, n_pt = pos.shape[1], pos.shape[0]
            n_data = inp.numel() if gather else out.numel()
            assert d_pos == (d_in if gather else d_out), "basis_rows: position table width"
        self._count("basis_rows")
        _check(self.lb.emu_basis_rows(_p(inp), d_in, _p(out), d_out, _p(ptr), _p(pt), _p(pos), d_pos, _p(meta),
                                      _p(coef), d_in, d_out, rows, n_pt, n_data, int(gather), int(scatter),
                                      int(inp.dtype == torch.float64)))

    # ---------------------------------------------------------------- radius graph
    @staticmethod
    def _grid(grid, ncell, periodic):
        assert len(grid) == 7 and len(ncell) == 3 and len(periodic) == 3 and min(ncell) >= 1
        return (ctypes.c_double * 7)(*grid), _i32(ncell), _i32(periodic)

    def radius_graph_cells(self, pos, grid, ncell, periodic, cell):
        assert pos.dtype == torch.float64 and cell.numel() == pos.shape[0]
        g, nc, pe = self._grid(grid, ncell, periodic)
        self._count("radius_graph_cells")
        _check(self.g.emu_radius_graph_cells(_p(pos), pos.shape[0], g, nc, pe, _p(cell)))

    def radius_graph_pass(self, pos, grid, ncell, periodic, targets, sorted_atoms, cell_start, counts, ptr, src,
                          vec):
        assert cell_start.numel() == ncell[0] * ncell[1] * ncell[2] + 1
        g, nc, pe = self._grid(grid, ncell, periodic)
        fill = ptr is not None
        assert (src is not None and vec is not None) if fill else counts is not None
        self._count("radius_graph_pass")
        _check(self.g.emu_radius_graph_pass(_p(pos), g, nc, pe, _p(targets), targets.numel(), _p(sorted_atoms),
                                            _p(cell_start), _p(counts), _p(ptr), _p(src), _p(vec), int(fill)))


def use_emulated_extension(monkeypatch, libs):
    """Route CPU tensors through the kernel path with :class:`EmulatedExtension` as the extension;
    returns the extension (its ``emulated_calls`` count the emulated launches)."""
    from maloq_b200 import ops
    from maloq_b200.ops import basis_transform, kernels, labels
    from maloq_b200.ops import loss as ops_loss

    ext = EmulatedExtension(libs)
    monkeypatch.setattr(kernels, "_lib", _Recorder(ext))
    for mod in (ops, ops_loss, labels, basis_transform):
        monkeypatch.setattr(mod, "_cuda", lambda *t: True)
    return ext
