"""A CPU stand-in for the compiled extension (``maloq_b200_C``), for tests.

Each function takes the same arguments as the extension's binding and writes the same outputs,
computed with PyTorch on CPU tensors from the contract stated in the kernel sources' comments
(``ops/csrc/*.cu``): GEMMs with bf16 operands and fp32 accumulation, the edge-frame gather /
rotate / rotate-back maps, the m-major gate, the norms, the fused loss.  Backward kernels are
the autograd gradients of the same definitions.  Per-CTA partial-sum outputs get the whole sum
in slice 0 and zeros elsewhere (the callers sum the slices).

With ``use_cpu_extension(monkeypatch)`` the op layer sends CPU tensors down the kernel path, so
the Python side of that path (views, strides, padding, buffer layouts, autograd functions,
weight caches, label rows) runs on a machine without a GPU and can be compared with the PyTorch
path.  The argument checks mirror the extension's (dtypes, shapes, contiguity, the 16-byte rule
of the TMA descriptors).  The peer-memory kernels (halo, barriers, fused all-reduce) work on
the host shared memory of ``tests/fake_symm.py``; the device radius graph is not provided.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def frame_rows(L, MM):
    """(degree, slot) of each m-major row of the (L, MM) edge frame: m = 0 rows l = 0..L (slot
    l), then for m = 1..min(MM, L) the +m rows and the -m rows of l = m..L, which share the
    slots base_m + l - m."""
    M = min(MM, L)
    ls, slots = list(range(L + 1)), list(range(L + 1))
    base = L + 1
    for m in range(1, M + 1):
        n = L - m + 1
        for _ in range(2):
            ls += list(range(m, L + 1))
            slots += list(range(base, base + n))
        base += n
    return ls, slots, base


def _bf(t):
    assert t.dtype == torch.bfloat16, t.dtype
    return t.float()


def _contig(*ts):
    for t in ts:
        assert t is None or t.is_contiguous(), "expected a contiguous tensor"


def _grad(fn, inputs, grad_out):
    """Gradients of fn(*inputs) w.r.t. the inputs that are not None (None for the others)."""
    leaves = [None if x is None else x.detach().float().requires_grad_(True) for x in inputs]
    with torch.enable_grad():  # called from inside autograd backward functions
        out = fn(*leaves)
        used = [x for x in leaves if x is not None]
        gs = torch.autograd.grad(out, used, grad_out, allow_unused=True)
    it = iter(gs)
    res = []
    for x in leaves:
        if x is None:
            res.append(None)
        else:
            g = next(it)
            res.append(torch.zeros_like(x) if g is None else g)
    return res


def _dst_of(dst_ptr, E):
    counts = dst_ptr[1:] - dst_ptr[:-1]
    dst = torch.repeat_interleave(torch.arange(len(counts)), counts)
    assert dst.numel() == E, "dst_ptr does not cover the edges"
    return dst


class CpuExtension:
    """The extension's bindings on CPU tensors (see the module docstring)."""

    def __init__(self, barrier_timeout=30.0):
        self._err = 0  # the device error word
        self.barrier_timeout = barrier_timeout  # seconds, the bounded spin of the device barriers

    # ------------------------------------------------------------------ GEMM
    def gemm(self, As, Bs, Cs, biases, mn, act, alpha, splits, bn, resids=()):
        assert 1 <= len(As) <= 8 and len(Bs) == len(Cs) == len(As)
        for i, (a, b, c) in enumerate(zip(As, Bs, Cs)):
            # the binding's checks, and the 16-byte rule of the TMA descriptors
            assert a.dtype == b.dtype == torch.bfloat16 and a.dim() == b.dim() == 2
            assert a.stride(1) == 1 and b.stride(1) == 1 and c.stride(-1) == 1
            assert c.dtype == Cs[0].dtype and c.dtype in (torch.float32, torch.bfloat16)
            M, K, N = (a.shape[1], a.shape[0], b.shape[1]) if mn else (a.shape[0], a.shape[1], b.shape[0])
            assert (b.shape[0] if mn else b.shape[1]) == K, "gemm: K mismatch"
            if splits > 1 or c.dim() == 3:
                assert c.dim() == 3 and c.dtype == torch.float32 and tuple(c.shape) == (splits, M, N)
            else:
                assert tuple(c.shape) == (M, N), (tuple(c.shape), M, N)
            for t in (a, b, c):
                assert t.data_ptr() % 16 == 0 and all((s * t.element_size()) % 16 == 0 for s in t.stride()[:-1])
            bias = biases[i] if i < len(biases) else None
            assert bias is None or (bias.dtype == torch.float32 and bias.numel() == N)
            res = resids[i] if i < len(resids) else None
            assert res is None or (res.dtype == torch.float32 and tuple(res.shape) == (M, N) and c.dtype == torch.float32)
            a, b = a.float(), b.float()
            if mn and c.dim() == 3:  # split-K over the rows: slice s takes rows s, s + splits, ...
                rows = torch.arange(a.shape[0])
                for s in range(c.shape[0]):
                    sel = rows[s::c.shape[0]]
                    c[s] = a[sel].T @ b[sel]
                continue
            y = a.T @ b if mn else alpha * (a @ b.T)
            if bias is not None:
                y = y + bias
            if act == 1:
                y = F.silu(y)
            if res is not None:
                y = y + res
            c.copy_(y.to(c.dtype))

    def weight_pack(self, srcs, dsts, kinds):
        from maloq_b200.ops import weights as W

        for S, D, k in zip(srcs, dsts, kinds):
            assert S.dtype == torch.float32 and S.is_contiguous() and D.is_contiguous()
            if k == 0:
                v = S
            elif k == 1:
                v = S.transpose(-1, -2)
            elif k == 2:
                v = W._pair(S)
            elif k == 3:
                v = W._pair(S).t()
            else:
                assert k == 4 and D.dtype == torch.float32
                v = W.pair_grad(S)
            assert D.numel() == v.numel()
            D.copy_(v.reshape(D.shape))

    def colsum_segments(self, X, seg, out):
        assert X.dim() == 2 and X.dtype == torch.float32 and out.is_contiguous()
        o = out.view(len(seg) - 1, X.shape[1])
        for s in range(len(seg) - 1):
            o[s] = X[seg[s]:seg[s + 1]].sum(0)

    def colsum(self, X, out):
        assert X.dim() == 2 and out.dtype == torch.float32 and out.numel() == X.shape[1]
        assert X.shape[1] <= 1 or X.stride(1) == 1
        out.copy_(X.float().sum(0))

    def splitk_reduce(self, part, out, beta):
        assert part.dtype == out.dtype == torch.float32 and out.is_contiguous()
        s = part.sum(0).view_as(out)
        out.copy_(s if beta == 0 else beta * out + s)  # beta = 0: out is not read (may be uninitialised)

    # ------------------------------------------------------------------ edge frame
    @staticmethod
    def _gather(L, MM, X, XE, src, dst, rot, rad, Cin):
        """A [E, R, Cin] (fp32) = rad[slot(k)] * rot . [X[src] | X[dst] | XE]."""
        ls, slots, ns = frame_rows(L, MM)
        E, R = src.shape[0], len(ls)
        parts = [X.index_select(0, src), X.index_select(0, dst)] + ([XE] if XE is not None else [])
        inp = torch.cat(parts, dim=2)[:, :, :Cin]
        u = torch.bmm(rot, inp)
        if rad is not None:
            u = u * rad.view(E, ns, Cin)[:, torch.tensor(slots)]
        return u

    def _extended(self, X, peers, halo_owner, halo_row, n_own):
        """[owned rows | halo rows read from their owners' staging slots]."""
        if peers == 0:
            return X
        SC = X[0].numel()
        halo = self._fetch_rows(peers, halo_owner, halo_row, SC).view(-1, *X.shape[1:])
        return torch.cat([X[:n_own], halo])

    def gather_rotate_fwd(self, L, MM, X, XE, src, dst, rot, rad, A, Cin, peers, halo_owner, halo_row, n_own):
        X = self._extended(X, peers, halo_owner, halo_row, n_own)
        _contig(X, XE, rot, A)
        assert X.dtype == rot.dtype == torch.float32 and A.dtype == torch.bfloat16
        E = src.shape[0]
        assert A.numel() == E * rot.shape[1] * Cin
        r = None if rad is None else _bf(rad)
        A.copy_(self._gather(L, MM, X, XE, src, dst, rot, r, Cin).reshape(A.shape).to(torch.bfloat16))

    def gather_rotate_bwd(self, L, MM, X, XE, rot, rad, dA, dst_ptr, src_perm, src_ptr, DX, DXE, DRAD, Cin,
                          peers=0, halo_owner=None, halo_row=None, n_own=0, recv=0, recv_slot=None):
        X = self._extended(X, peers, halo_owner, halo_row, n_own)
        E = rot.shape[0]
        N = DX.shape[0]
        assert dst_ptr.numel() == N + 1 and src_ptr.numel() == N + 1
        dst = _dst_of(dst_ptr, E)
        # the sources from the source CSR: edge src_perm[i] has source n for i in [ptr[n], ptr[n+1])
        src = torch.empty(E, dtype=torch.long)
        src[src_perm] = _dst_of(src_ptr, E)
        R = rot.shape[1]
        g = _bf(dA).view(E, R, Cin)
        r = None if rad is None else _bf(rad)
        gx, gxe, grad_r = _grad(lambda x, xe, rr: self._gather(L, MM, x, xe, src, dst, rot, rr, Cin), [X, XE, r], g)
        if recv:  # halo rows into their owners' receive slots, owned rows into DX
            from tests.fake_symm import floats_at, table

            assert peers and recv_slot is not None
            SC = gx[0].numel()
            bases = table(recv, self._world())
            for h, (o, sl) in enumerate(zip(halo_owner, recv_slot)):
                floats_at(bases[int(o)] + 4 * int(sl) * SC, SC).copy_(gx[n_own + h].reshape(-1))
            DX[:n_own].copy_(gx[:n_own])
        else:
            DX.copy_(gx[:N])
        if DXE is not None:
            DXE.copy_(gxe)
        if DRAD is not None:
            DRAD.copy_(grad_r.to(torch.bfloat16))

    @staticmethod
    def _rotate_back(Y, koff, Rk, rot, C):
        E = rot.shape[0]
        y = _bf(Y)[:, koff:koff + Rk * C].reshape(E, Rk, C)
        return torch.bmm(rot[:, :Rk].transpose(1, 2), y)

    def rotate_back_scatter(self, L, MM, Y, koff, Rk, rot, dst_ptr, base, out, scale):
        assert out.dtype == torch.float32 and out.is_contiguous()
        E = rot.shape[0]
        msg = self._rotate_back(Y, koff, Rk, rot, out.shape[2])
        acc = torch.zeros_like(out).index_add_(0, _dst_of(dst_ptr, E), msg) * scale
        out.copy_(acc + (base if base is not None else 0.0))

    def rotate_back_edge(self, L, MM, Y, koff, Rk, rot, out):
        assert out.dtype == torch.float32 and out.is_contiguous()
        out.copy_(self._rotate_back(Y, koff, Rk, rot, out.shape[2]))

    def rotate_grad(self, L, MM, G, rows, rot, DY, DYf, Rk, scale):
        E, C = rot.shape[0], G.shape[2]
        g = G.index_select(0, rows) if rows is not None else G
        d = (scale * torch.bmm(rot[:, :Rk], g)).reshape(E, Rk * C)
        for t in (DY, DYf):
            if t is not None:
                t[:, :Rk * C].copy_(d.to(t.dtype))

    @staticmethod
    def _gate(L, MM, y1, H):
        ls, _, _ = frame_rows(L, MM)
        E, G = y1.shape[0], L * H
        g = torch.tanh(y1[:, :G].reshape(E, L, H))
        x = y1[:, G:].reshape(E, len(ls), H)
        rows = [F.silu(x[:, 0])] + [x[:, k] * g[:, l - 1] for k, l in enumerate(ls) if k > 0]
        return torch.stack(rows, 1).reshape(E, -1)

    def gate_fwd(self, L, MM, Y1, H1, H):
        H1.copy_(self._gate(L, MM, _bf(Y1), H).to(torch.bfloat16))

    def gate_bwd(self, L, MM, Y1, dH1, dY1, H):
        (g,) = _grad(lambda y: self._gate(L, MM, y, H), [_bf(Y1)], _bf(dH1))
        dY1.copy_(g.to(torch.bfloat16))

    # ------------------------------------------------------------------ norms and gates
    @staticmethod
    def _rms(L, s, aw, ab, eps):
        from maloq_b200.ops import reference as R

        S = (L + 1) ** 2
        bw = torch.zeros(S, 1)
        for l in range(L + 1):
            bw[l * l:(l + 1) ** 2] = 1.0 / ((2 * l + 1) * (L + 1))
        return R.rms_norm_sh(s, aw, ab, bw, eps)

    def norm_grid(self, rows):
        return 1

    def rms_norm_fwd(self, L, X, RES, aw, ab, OUT, SUM, eps):
        _contig(X, RES, OUT, SUM)
        s = X + RES if RES is not None else X
        if SUM is not None:
            SUM.copy_(s)
        OUT.copy_(self._rms(L, s, aw, ab, eps).to(OUT.dtype))

    def rms_norm_bwd(self, L, Sx, G, GS, aw, DX, PART, eps):
        ab = torch.zeros(aw.shape[1])
        gx, gw, gb = _grad(lambda s, w, b: self._rms(L, s, w, b, eps), [Sx, aw, ab], G.float())
        DX.copy_(gx + (GS if GS is not None else 0.0))
        PART.zero_()
        PART[0, :L + 1] = gw
        PART[0, L + 1] = gb

    def ln_silu_fwd(self, X, w, b, OUT, eps):
        OUT.copy_(F.silu(F.layer_norm(X, (X.shape[1],), w, b, eps)).to(OUT.dtype))

    def ln_silu_bwd(self, X, w, b, G, DX, PART, eps):
        gx, gw, gb = _grad(lambda x, ww, bb: F.silu(F.layer_norm(x, (x.shape[1],), ww, bb, eps)), [X, w, b], _bf(G))
        DX.copy_(gx)
        PART.zero_()
        PART[0, 0] = gw
        PART[0, 1] = gb

    @staticmethod
    def _gate_l(L, x, gt):
        B, S, H = x.shape
        t = torch.tanh(gt.view(B, L, H))
        rows = [F.silu(x[:, :1])] + [x[:, l * l:(l + 1) ** 2] * t[:, l - 1:l] for l in range(1, L + 1)]
        return torch.cat(rows, 1)

    def gate_l_fwd(self, L, X, Gt, OUT, silu_gates=False):
        OUT.copy_(self._gate_l(L, X.float(), F.silu(Gt) if silu_gates else Gt).to(OUT.dtype))

    def gate_l_bwd(self, L, X, Gt, DO, DX, DG, silu_gates=False):
        gx, gg = _grad(lambda x, g: self._gate_l(L, x, F.silu(g) if silu_gates else g), [X.float(), Gt],
                       DO.float())
        DX.copy_(gx.to(DX.dtype))
        DG.copy_(gg)

    @staticmethod
    def _head_gate(L, x, sv, act, scale, absg):
        B, S, C = x.shape
        u = sv[:, C:].reshape(B, L, C)
        u = u.abs() if absg else u
        g = (torch.sigmoid(u) if act == 0 else torch.tanh(u)) * scale
        rows = [sv[:, :C].unsqueeze(1)] + [x[:, l * l:(l + 1) ** 2] * g[:, l - 1:l] for l in range(1, L + 1)]
        return torch.cat(rows, 1)

    def head_gate_fwd(self, L, X, SV, A, act, scale, absg):
        assert A.dtype == torch.bfloat16 and A.shape == X.shape and SV.shape == (X.shape[0], (L + 1) * X.shape[2])
        A.copy_(self._head_gate(L, X, SV, act, scale, absg).to(torch.bfloat16))

    def head_gate_bwd(self, L, X, SV, DA, DX, DSV, act, scale, absg):
        gx, gs = _grad(lambda x, s: self._head_gate(L, x, s, act, scale, absg), [X, SV], DA)
        DX.copy_(gx)
        DSV.copy_(gs)

    def edge_inputs(self, src_z, dst_z, edge_attr, src_table, dst_table, offset, coeff, OUT):
        C, NB = src_table.shape[1], offset.numel()
        assert OUT.dtype == torch.bfloat16 and tuple(OUT.shape) == (src_z.numel(), 2 * C + NB)
        g = torch.exp(coeff * (edge_attr[:, 0:1] - offset.view(1, -1)) ** 2)
        OUT.copy_(torch.cat([src_table[src_z], g, dst_table[dst_z]], 1).to(torch.bfloat16))

    # ------------------------------------------------------------------ label rows
    def basis_rows(self, inp, out, ptr, pt, pos, meta, coef, d_in, rows, gather, scatter):
        """out[r, u] = sum_{j < n_u} in[r, s_u + j] * coef[c_u + j n_u], meta[u] = (s_u, n_u, c_u, 0);
        gather: in[r, k] = data[ptr[r] + pos[pt[r], k]] (0 where pos < 0); scatter: data[ptr[r] +
        pos[pt[r], u]] = out[r, u] (skipped where pos < 0); otherwise dense rows."""
        assert inp.dtype == out.dtype == coef.dtype and inp.dtype in (torch.float32, torch.float64)
        assert meta.dtype == torch.int32 and meta.shape[1] == 4
        d_out = meta.shape[0]
        if gather:
            p = pos[pt[:rows]].long()  # [rows, d_in]
            idx = ptr[:rows, None] + p.clamp(min=0)
            x = torch.where(p >= 0, inp.reshape(-1)[idx], torch.zeros((), dtype=inp.dtype))
        else:
            x = inp.reshape(-1)[: rows * d_in].view(rows, d_in)
        y = torch.empty(rows, d_out, dtype=inp.dtype)
        for u in range(d_out):
            su, nu, cu = (int(v) for v in meta[u, :3])
            c = coef[cu + torch.arange(nu) * nu]
            y[:, u] = x[:, su:su + nu] @ c
        if scatter:
            p = pos[pt[:rows]].long()  # [rows, d_out]
            ok = p >= 0
            flat = out.view(-1)
            flat[(ptr[:rows, None] + p)[ok]] = y[ok]
        else:
            out.view(-1)[: rows * d_out].copy_(y.reshape(-1))

    # ------------------------------------------------------------------ rotation, loss, status
    def edge_rotation(self, vec, J, joff, L, row_l, row_m, ROT):
        from maloq_b200.core import sph

        Js = [J[joff[l]:joff[l] + (2 * l + 1) ** 2].view(2 * l + 1, 2 * l + 1) for l in range(L + 1)]
        alpha, beta = sph.edge_euler_angles(vec.double())
        D = sph.block_diag_wigner(L, torch.zeros_like(alpha), -beta, -alpha, [j.double() for j in Js])
        idx = torch.tensor([l * l + l + m for l, m in zip(row_l, row_m)])
        ROT.copy_(D.index_select(1, idx).float())

    def fock_loss_grid(self, n):
        return 1

    def fock_loss_stats(self, O, T, pt, mask, part):
        m = mask[pt].float()
        d = O - T
        part.zero_()
        part[0] = torch.stack([(m * d * d).sum(), (m * d.abs()).sum(), m.sum()])

    def fock_loss_grad(self, O, T, pt, mask, gstat, G):
        m = mask[pt].float()
        d = O - T
        G.copy_(m * (gstat[0] * 2 * d + gstat[1] * torch.sign(d)))

    def error_status(self, clear):
        e = self._err
        if clear:
            self._err = 0
        return e

    # ------------------------------------------------------------------ peer memory
    # (addresses from tests/fake_symm.py: every rank's buffers mapped into this process)
    @staticmethod
    def _world():
        import torch.distributed as dist

        return dist.get_world_size() if dist.is_initialized() else 1

    def _barrier(self, pads_dev, rank, world, epoch, slot_base, mask):
        import time

        from tests.fake_symm import PAD_WORDS, int32_at, table

        pads = table(pads_dev, world)
        members = [t for t in range(world) if mask == 0 or (mask >> t) & 1 or t == rank]
        for t in members:
            int32_at(pads[t], PAD_WORDS)[slot_base + rank] = epoch
        mine = int32_at(pads[rank], PAD_WORDS)
        deadline = time.time() + self.barrier_timeout
        for t in members:
            while int(mine[slot_base + t]) - epoch < 0:
                if time.time() > deadline:
                    self._err = self._err or 4  # a peer did not arrive
                    return
                time.sleep(2e-4)

    def peer_barrier(self, pads_dev, rank, world, epoch, slot_base, spin_limit):
        self._barrier(pads_dev, rank, world, epoch, slot_base, 0)

    def peer_barrier_mask(self, pads_dev, rank, world, epoch, slot_base, spin_limit, mask):
        assert mask != 0
        self._barrier(pads_dev, rank, world, epoch, slot_base, mask & ((1 << 64) - 1))

    def allreduce_p2p(self, bufs_dev, rank, world, off, n, scale):
        """Rank r reduces chunk r over all ranks' buffers and writes it back into every one."""
        from tests.fake_symm import floats_at, table

        chunk = ((n + world - 1) // world + 3) // 4 * 4
        c0, c1 = off + rank * chunk, min(off + (rank + 1) * chunk, off + n)
        if c1 <= c0:
            return
        views = [floats_at(b + 4 * c0, c1 - c0) for b in table(bufs_dev, world)]
        total = torch.stack([v.clone() for v in views]).sum(0) * scale
        for v in views:
            v.copy_(total)

    def _fetch_rows(self, peers, halo_owner, halo_row, SC):
        from tests.fake_symm import floats_at, table

        bases = table(peers, self._world())
        rows = [floats_at(bases[int(o)] + 4 * int(r) * SC, SC).clone() for o, r in zip(halo_owner, halo_row)]
        return torch.stack(rows) if rows else torch.zeros(0, SC)

    def halo_fetch(self, peers, halo_owner, halo_row, OUT):
        SC = OUT[0].numel() if OUT.shape[0] else 0
        if OUT.shape[0]:
            OUT.view(OUT.shape[0], SC).copy_(self._fetch_rows(peers, halo_owner, halo_row, SC))

    def halo_push(self, G, recv, halo_owner, recv_slot):
        from tests.fake_symm import floats_at, table

        SC = G.shape[1]
        bases = table(recv, self._world())
        for h, (o, sl) in enumerate(zip(halo_owner, recv_slot)):
            floats_at(bases[int(o)] + 4 * int(sl) * SC, SC).copy_(G[h])

    def node_reduce(self, DDST, dst_ptr, DSRC, src_perm, src_ptr, DX):
        N = DX.shape[0]
        out = torch.zeros(N, DX[0].numel() if N else 0)
        if DDST is not None:
            out.index_add_(0, _dst_of(dst_ptr, DDST.shape[0]), DDST.reshape(DDST.shape[0], -1))
        if DSRC is not None:
            rows = _dst_of(src_ptr, src_perm.numel())
            out.index_add_(0, rows, DSRC.reshape(DSRC.shape[0], -1)[src_perm])
        DX.view(N, -1).copy_(out)

    def bounds_checked(self):
        return False


class _Recorder:
    """Delegates to the stand-in and records which bindings were called (``calls``)."""

    def __init__(self, ext):
        self._ext, self.calls = ext, {}

    def __getattr__(self, name):
        fn = getattr(self._ext, name)

        def call(*a, **k):
            self.calls[name] = self.calls.get(name, 0) + 1
            return fn(*a, **k)

        return call


def use_cpu_extension(monkeypatch):
    """Route CPU tensors through the kernel path with :class:`CpuExtension` as the extension."""
    from maloq_b200 import ops
    from maloq_b200.ops import kernels

    ext = _Recorder(CpuExtension())
    monkeypatch.setattr(kernels, "_lib", ext)
    from maloq_b200.ops import basis_transform, labels
    from maloq_b200.ops import loss as ops_loss

    # every module that decides CPU vs kernel path with _cuda
    for mod in (ops, ops_loss, labels, basis_transform):
        monkeypatch.setattr(mod, "_cuda", lambda *t: True)
    return ext
