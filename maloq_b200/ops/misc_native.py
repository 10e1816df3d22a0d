"""Kernel-backed edge rotation construction and fused masked Fock loss."""

from __future__ import annotations

import torch

from .native import count_launches


def _lib():
    from .kernels import lib

    return lib()


def _colsum(x):
    from .kernels import colsum

    return colsum(x)


_J_CACHE = {}


def edge_rotation(vec_yzx, lmax, mmax, Js, mapping):
    """rot [E, R, (L+1)^2]: m-major rows |m| <= mmax of D(0, -beta, -alpha) (no gradient)."""
    dev = vec_yzx.device
    key = (dev, lmax, mmax, id(Js[0]))
    if key not in _J_CACHE:
        flat = torch.cat([J.reshape(-1).float() for J in Js[: lmax + 1]]).to(dev).contiguous()
        joff, o = [], 0
        for l in range(lmax + 1):
            joff.append(o)
            o += (2 * l + 1) ** 2
        ls = mapping.l_harmonic.tolist()
        ms = mapping.m_complex.tolist()
        _J_CACHE[key] = (flat, joff, ls, ms)
    flat, joff, ls, ms = _J_CACHE[key]
    v = vec_yzx.detach().float().contiguous()
    E = v.shape[0]
    rot = torch.empty(E, len(ls), (lmax + 1) ** 2, device=dev, dtype=torch.float32)
    _lib().edge_rotation(v, flat, joff, lmax, ls, ms, rot)
    count_launches(1)
    return rot


class _LossStats(torch.autograd.Function):
    @staticmethod
    def forward(ctx, no, eo, nt, et, mask, npt, ept):
        lib = _lib()
        no, eo = no.contiguous().float(), eo.contiguous().float()
        nt, et = nt.contiguous().float(), et.contiguous().float()
        out = []
        for o, t, pt in ((no, nt, npt), (eo, et, ept)):
            grid = lib.fock_loss_grid(o.numel())
            part = torch.empty(grid, 3, device=o.device, dtype=torch.float32)
            lib.fock_loss_stats(o, t, pt, mask, part)
            out.append(_colsum(part))
        count_launches(2)
        ctx.save_for_backward(no, eo, nt, et, mask, npt, ept)
        return torch.cat(out)

    @staticmethod
    def backward(ctx, g):
        lib = _lib()
        no, eo, nt, et, mask, npt, ept = ctx.saved_tensors
        g = g.float().contiguous()  # stays on the device: no host sync in the backward
        gn = torch.empty_like(no)
        ge = torch.empty_like(eo)
        lib.fock_loss_grad(no, nt, npt, mask, g[0:2], gn)
        lib.fock_loss_grad(eo, et, ept, mask, g[3:5], ge)
        count_launches(2)
        return gn, ge, None, None, None, None, None


def fock_loss(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt, name):
    """(node loss, edge loss, total loss) of a decomposable loss from the fused statistics."""
    from .loss import DECOMPOSABLE

    f = DECOMPOSABLE[name]
    mask = mask_table.to(device=node_out.device, dtype=torch.uint8).contiguous()
    st = _LossStats.apply(node_out, edge_out, node_t, edge_t, mask, node_pt.contiguous(), edge_pt.contiguous())
    sse_n, sae_n, cnt_n, sse_e, sae_e, cnt_e = st.unbind(0)
    ln = f(sse_n / cnt_n, sae_n / cnt_n)
    le = f(sse_e / cnt_e, sae_e / cnt_e)
    ct = cnt_n + cnt_e
    lt = f((sse_n + sse_e) / ct, (sae_n + sae_e) / ct)
    return ln, le, lt


class _EdgeInputs(torch.autograd.Function):
    """Radial-MLP input rows [E, 2C + NB] bf16 in one kernel: source-element embedding,
    Gaussian expansion of the edge length, target-element embedding.  Backward: the two
    embedding tables' gradients as one-hot GEMMs (the Gaussian part has no parameters)."""

    @staticmethod
    def forward(ctx, src_z, dst_z, edge_attr, src_w, dst_w, offset, coeff):
        E, C, NB = src_z.shape[0], src_w.shape[1], offset.numel()
        out = torch.empty(E, 2 * C + NB, device=src_w.device, dtype=torch.bfloat16)
        _lib().edge_inputs(src_z.contiguous(), dst_z.contiguous(), edge_attr.contiguous().float(),
                           src_w.detach().contiguous().float(), dst_w.detach().contiguous().float(),
                           offset.contiguous().float(), float(coeff), out)
        count_launches(1)
        ctx.save_for_backward(src_z, dst_z)
        ctx.dims = (C, NB, src_w.shape[0], dst_w.shape[0])
        return out

    @staticmethod
    def backward(ctx, g):
        src_z, dst_z = ctx.saved_tensors
        C, NB, ns, nd = ctx.dims
        g = g.float()
        gs = gd = None
        if ctx.needs_input_grad[3]:
            oh = (src_z.unsqueeze(1) == torch.arange(ns, device=g.device)).to(g.dtype)
            gs = oh.t() @ g[:, :C]
        if ctx.needs_input_grad[4]:
            oh = (dst_z.unsqueeze(1) == torch.arange(nd, device=g.device)).to(g.dtype)
            gd = oh.t() @ g[:, C + NB:]
        return None, None, None, gs, gd, None, None


def edge_inputs(src_z, dst_z, edge_attr, src_w, dst_w, offset, coeff):
    return _EdgeInputs.apply(src_z, dst_z, edge_attr, src_w, dst_w, offset, coeff)
