"""Edgewise message pass on the kernel library (forward and backward).

Forward (per layer, node or edge path):

1. ``gather_rotate_fwd``: A = rad * rot . [x[src] | x[dst] (| x_edge)] -> bf16 [E, R*Cin]
   (rad: the radial MLP's output, bf16 [E, NS*Cin])
2. grouped tcgen05 GEMM, one problem per |m| (pair weights for m > 0) -> Y1 = [gates | m-major]
3. ``gate_fwd`` -> H1 [E, R*H]
4. grouped tcgen05 GEMM (second SO(2) conv) -> Y2 [E, R*C]
5. ``rotate_back_scatter`` (node path, fixed-order sum over each node's incoming edges) or
   ``rotate_back_edge`` (edge path).

Backward runs the transposed chain; weight gradients are deterministic split-K GEMMs over
the edges; node gradients come out of one kernel that walks each node's incoming and
outgoing edges in a fixed order and recomputes their contributions from dA (no per-edge
gradient rows).
Reference: ``helm/esen_block.py:146-258`` and ``helm/nn/so2_layers.py:139-214``.
"""

from __future__ import annotations

import torch

from . import weights as W
from .native import count_launches


def _lib():
    from .kernels import lib

    return lib()


def _colsum(x):
    from .kernels import colsum

    return colsum(x)


def dst_ptr_ext(graph, n):
    """Destination CSR offsets over ``n`` rows (halo rows, beyond the owned ones, have no
    incoming edges)."""
    if n == graph.dst_ptr.shape[0] - 1:
        return graph.dst_ptr
    key = ("dst_ptr_ext", n)
    if key not in graph.cache:
        tail = graph.dst_ptr[-1:].expand(n + 1 - graph.dst_ptr.shape[0])
        graph.cache[key] = torch.cat([graph.dst_ptr, tail]).contiguous()
    return graph.cache[key]


def src_csr(graph):
    """Edges grouped by source node: (perm, ptr), cached on the graph."""
    key = "src_csr"
    if key not in graph.cache:
        src = graph.src
        n = graph.num_nodes_ext if hasattr(graph, "num_nodes_ext") else graph.num_nodes
        perm = torch.argsort(src, stable=True)
        # ptr[i] = number of edges with source < i: a search in the sorted sources, which (unlike
        # a bincount) needs no device-to-host read of the largest index
        ptr = torch.searchsorted(src[perm], torch.arange(n + 1, device=src.device, dtype=src.dtype))
        graph.cache[key] = (perm, ptr)
    return graph.cache[key]


# ------------------------------------------------------------------ grouped GEMM helpers
def _blocks(m_size, width, extra=0):
    """Column ranges [(c0, c1)] of each |m| block in a row of R*width (+extra leading) values."""
    out, off = [], 0
    for m, ms in enumerate(m_size):
        n = ms if m == 0 else 2 * ms
        if m == 0:
            out.append((0, extra + n * width))
            off = extra + n * width
        else:
            out.append((off, off + n * width))
            off += n * width
    return out


def _gemm(As, Ws, Cs, biases, bn=128):
    _lib().gemm(As, Ws, Cs, biases, False, 0, 1.0, 1, bn)
    count_launches(1)


def _weight_grads(gys, xs):
    """[gy_i^T @ x_i] for each problem, one grouped split-K launch + reductions."""
    M = gys[0].shape[0]
    tiles = sum(((g.shape[1] + 127) // 128) * ((x.shape[1] + 127) // 128) for g, x in zip(gys, xs))
    splits = max(1, min(-(-296 // tiles), M // 2048, 32))
    outs = [torch.empty(g.shape[1], x.shape[1], device=g.device, dtype=torch.float32) for g, x in zip(gys, xs)]
    if M == 0:
        return [o.zero_() for o in outs]
    if splits == 1:
        _lib().gemm(gys, xs, outs, [None] * len(gys), True, 0, 1.0, 1, 128)
        count_launches(1)
        return outs
    parts = [torch.empty(splits, g.shape[1], x.shape[1], device=g.device, dtype=torch.float32) for g, x in zip(gys, xs)]
    _lib().gemm(gys, xs, parts, [None] * len(gys), True, 0, 1.0, splits, 128)
    for p, o in zip(parts, outs):
        _lib().splitk_reduce(p, o, 0.0)
    count_launches(1 + len(parts))
    return outs


class EdgewiseFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_node, x_edge_emb, rad, b1, b2, graph, meta, halo, *weights):
        """``weights``: fc_m0.weight and the SO2_m_Conv fc.weight of each |m| > 0 (the pair
        matrices are built from them in the bf16 weight cache) for both convolutions."""
        lib = _lib()
        nw = len(weights) // 2
        w1, w2 = weights[:nw], weights[nw:]
        S, C = x_node.shape[1], x_node.shape[2]
        R, H, L, Cin, G = meta["R"], meta["H"], meta["L"], meta["Cin"], meta["G"]
        LM = (meta["L"], meta["MM"])
        E = graph.src.shape[0]
        dev = x_node.device
        x_node = x_node.contiguous()
        xe = x_edge_emb.contiguous() if x_edge_emb is not None else None
        rad = rad.to(torch.bfloat16).contiguous()
        A = torch.empty(E, R * Cin, device=dev, dtype=torch.bfloat16)
        lib.gather_rotate_fwd(*LM, x_node, xe, graph.src, graph.dst, graph.rot, rad, A, Cin, *_halo_args(halo))
        w1b = [W.bf16(w1[0])] + [W.pair_bf16(w) for w in w1[1:]]
        w2b = [W.bf16(w2[0])] + [W.pair_bf16(w) for w in w2[1:]]
        Y1 = torch.empty(E, G + R * H, device=dev, dtype=torch.bfloat16)
        ab = _blocks(meta["m_size"], Cin)
        yb = _blocks(meta["m_size"], H, G)
        _gemm([A[:, a0:a1] for a0, a1 in ab], w1b, [Y1[:, y0:y1] for y0, y1 in yb],
              [b1.float().contiguous()] + [None] * (nw - 1))
        H1 = torch.empty(E, R * H, device=dev, dtype=torch.bfloat16)
        lib.gate_fwd(*LM, Y1, H1, H)
        Co = meta["Co"]  # output channels of the second convolution (C, or a padded head width)
        Y2 = torch.empty(E, R * Co, device=dev, dtype=torch.bfloat16)
        hb = _blocks(meta["m_size"], H)
        cb = _blocks(meta["m_size"], Co)
        _gemm([H1[:, a0:a1] for a0, a1 in hb], w2b, [Y2[:, y0:y1] for y0, y1 in cb],
              [b2.float().contiguous()] + [None] * (nw - 1))
        if meta["node"]:
            # rows of the destination range (all nodes, or one chunk's nodes)
            out = torch.empty(graph.num_out, S, Co, device=dev, dtype=torch.float32)
            lib.rotate_back_scatter(*LM, Y2, 0, R, graph.rot, graph.out_ptr, None, out, 1.0)
        else:
            out = torch.empty(E, S, Co, device=dev, dtype=torch.float32)
            lib.rotate_back_edge(*LM, Y2, 0, R, graph.rot, out)
        count_launches(4)
        ctx.save_for_backward(x_node, xe, rad, A, Y1, H1, *weights)
        ctx.graph, ctx.meta, ctx.nw, ctx.halo = graph, meta, nw, halo
        return out

    @staticmethod
    def backward(ctx, g):
        lib = _lib()
        graph, meta, nw = ctx.graph, ctx.meta, ctx.nw
        saved = ctx.saved_tensors
        x_node, xe, rad, A, Y1, H1 = saved[:6]
        w1, w2 = saved[6:6 + nw], saved[6 + nw:]
        w1t = [W.bf16_t(w1[0])] + [W.pair_bf16_t(w) for w in w1[1:]]
        w2t = [W.bf16_t(w2[0])] + [W.pair_bf16_t(w) for w in w2[1:]]
        S, C = x_node.shape[1], x_node.shape[2]
        R, H, L, Cin, G = meta["R"], meta["H"], meta["L"], meta["Cin"], meta["G"]
        LM = (meta["L"], meta["MM"])
        E = graph.src.shape[0]
        dev = g.device
        g = g.contiguous().float()
        Co = meta["Co"]
        dY2 = torch.empty(E, R * Co, device=dev, dtype=torch.bfloat16)
        _rotate_grad(LM, g, graph, meta["node"], dY2, None, R, 1.0)
        hb = _blocks(meta["m_size"], H)
        cb = _blocks(meta["m_size"], Co)
        ab = _blocks(meta["m_size"], Cin)
        yb = _blocks(meta["m_size"], H, G)
        # conv2
        dH1 = torch.empty(E, R * H, device=dev, dtype=torch.bfloat16)
        _gemm([dY2[:, a0:a1] for a0, a1 in cb], w2t, [dH1[:, h0:h1] for h0, h1 in hb], [None] * nw)
        dw2 = _weight_grads([dY2[:, a0:a1] for a0, a1 in cb], [H1[:, h0:h1] for h0, h1 in hb])
        db2 = _colsum(dY2[:, cb[0][0]:cb[0][1]])
        # gate
        dY1 = torch.empty_like(Y1)
        lib.gate_bwd(*LM, Y1, dH1, dY1, H)
        # conv1
        dA = torch.empty(E, R * Cin, device=dev, dtype=torch.bfloat16)
        _gemm([dY1[:, y0:y1] for y0, y1 in yb], w1t, [dA[:, a0:a1] for a0, a1 in ab], [None] * nw)
        dw1 = _weight_grads([dY1[:, y0:y1] for y0, y1 in yb], [A[:, a0:a1] for a0, a1 in ab])
        db1 = _colsum(dY1[:, yb[0][0]:yb[0][1]])
        # gather: node gradients straight from dA (fixed-order walks over each node's incoming
        # and outgoing edges), the edge-embedding part per edge, the radial gradient per edge
        perm, sptr = src_csr(graph)
        n_ext = graph.num_nodes_ext if ctx.halo is not None else x_node.shape[0]
        DX = torch.empty((n_ext,) + tuple(x_node.shape[1:]), device=dev, dtype=torch.float32)
        DXE = torch.empty_like(xe) if xe is not None else None
        DRAD = torch.empty_like(rad)
        if ctx.halo is not None:  # halo rows' gradients go straight to their owners' receive slots
            peer = ctx.halo[0]
            b, recv = peer.begin_grads()
            lib.gather_rotate_bwd(*LM, x_node, xe, graph.rot, rad, dA, dst_ptr_ext(graph, n_ext), perm, sptr, DX,
                                  DXE, DRAD, Cin, *_halo_args(ctx.halo), recv, peer.recv_slot)
            DX = peer.finish_grads(DX[:peer.n_own], b)
        else:
            lib.gather_rotate_bwd(*LM, x_node, xe, graph.rot, rad, dA, dst_ptr_ext(graph, n_ext), perm, sptr, DX,
                                  DXE, DRAD, Cin, *_halo_args(ctx.halo))
        count_launches(5 + (xe is not None))
        pg = W.pair_grads(dw1[1:] + dw2[1:])
        dw1 = dw1[:1] + pg[:nw - 1]
        dw2 = dw2[:1] + pg[nw - 1:]
        return (DX, DXE, DRAD, db1, db2, None, None, None, *dw1, *dw2)


def edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge):
    c1, c2 = mod.so2_conv_1, mod.so2_conv_2
    mapping = mod.mapping
    C = x_node.shape[2]
    Cin = mod.concat_size * C
    key = ("edge_meta", id(mod), node_or_edge)
    meta = graph.cache.get(key)
    co = c2.m_output_channels
    cp = co if co % 8 == 0 else (co + 7) // 8 * 8  # GEMM / rotate-back rows: 16-byte aligned widths
    if meta is None:
        meta = dict(R=mapping.res_size, H=c1.m_output_channels, L=mod.lmax, MM=mod.mmax, Cin=Cin,
                    G=c1.extra_m0_output_channels, m_size=list(mapping.m_size), node=node_or_edge == "node", Co=cp)
        graph.cache[key] = meta
    rad = c1.rad_func(x_edge, out_dtype=torch.bfloat16)
    halo = None
    x_src_space = x_node
    if graph.halo is not None:
        if graph.halo.transport == "peer":
            peer = graph.halo.peer_for(tuple(x_node.shape[1:]))
            halo = (peer, peer.publish(x_node))  # rows readable by every rank; slot id
        else:
            x_src_space = graph.halo.extend(x_node, graph)
    w2 = [c2.fc_m0.weight] + [c.fc.weight for c in c2.so2_m_conv]
    b2 = c2.fc_m0.bias
    if cp != co:
        # narrow heads (e.g. one force channel): zero output channels up to cp, as differentiable
        # views of the parameters (their gradients come back unpadded); the caller sees co channels
        w2 = [_pad_out_channels(w, co, cp) for w in w2]
        b2 = _pad_out_channels(b2, co, cp)
    weights = [c1.fc_m0.weight] + [c.fc.weight for c in c1.so2_m_conv] + w2
    out = EdgewiseFn.apply(x_src_space, x_msg_edge, rad, c1.fc_m0.bias, b2, graph, meta, halo, *weights)
    return out if cp == co else out[..., :co]


def _pad_out_channels(w, co, cp):
    """Rows of a convolution weight (or bias) grouped as [..., co] output channels -> cp
    channels, the new ones zero: [n*co, K] -> [n*cp, K] (and [n*co] -> [n*cp])."""
    if w.dim() == 1:
        return torch.nn.functional.pad(w.view(-1, co), (0, cp - co)).reshape(-1)
    return torch.nn.functional.pad(w.view(-1, co, w.shape[1]), (0, 0, 0, cp - co)).reshape(-1, w.shape[1])


def _rotate_grad(LM, g, graph, node, DY, DYf, Rk, scale):
    """Backward of rotate-back, edge-parallel: node path reads each edge's destination row of
    the gradient (``dst_out``), the edge path its own row.  (Walking each destination's edge
    range instead leaves too few CTAs at molecular node counts.)"""
    _lib().rotate_grad(*LM, g, graph.dst_out if node else None, graph.rot, DY, DYf, Rk, scale)


def _halo_args(halo):
    """(peer pointer table, halo owner, halo row, n_own) for the gather kernels."""
    if halo is None:
        return 0, None, None, 0
    peer, slot = halo
    return peer.table_ptr(slot), peer.halo_owner, peer.halo_row, peer.n_own


class RotateBackM0Fn(torch.autograd.Function):
    """m = 0 coefficients [E, n0, C] rotated back to the node frame: summed into ``base``
    per destination node (times ``scale``), or returned per edge when ``base`` is None."""

    @staticmethod
    def forward(ctx, e, base, graph, scale):
        lib = _lib()
        E, n0, C = e.shape
        S = (graph.lmax + 1) ** 2
        Y = e.reshape(E, n0 * C).to(torch.bfloat16).contiguous()
        if base is not None:
            out = torch.empty(graph.num_out, S, C, device=e.device, dtype=torch.float32)
            lib.rotate_back_scatter(graph.lmax, graph.mmax, Y, 0, n0, graph.rot, graph.out_ptr,
                                    base.contiguous().float(), out, scale)
        else:
            out = torch.empty(E, S, C, device=e.device, dtype=torch.float32)
            lib.rotate_back_edge(graph.lmax, graph.mmax, Y, 0, n0, graph.rot, out)
        count_launches(1)
        ctx.graph, ctx.scale, ctx.n0, ctx.node = graph, scale, n0, base is not None
        return out

    @staticmethod
    def backward(ctx, g):
        graph = ctx.graph
        g = g.contiguous().float()
        E = graph.src.shape[0]
        C = g.shape[2]
        de = torch.empty(E, ctx.n0 * C, device=g.device, dtype=torch.float32)
        _rotate_grad((graph.lmax, graph.mmax), g, graph, ctx.node, None, de, ctx.n0, ctx.scale if ctx.node else 1.0)
        count_launches(1)
        return de.view(E, ctx.n0, C), (g if ctx.node else None), None, None


def rotate_back_m0(e, graph, base=None, scale=1.0):
    return RotateBackM0Fn.apply(e, base, graph, float(scale))
