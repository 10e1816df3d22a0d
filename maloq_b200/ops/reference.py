"""PyTorch definitions of every op (the CPU path and the oracle for the CUDA kernels).

Each function restates the reference math in plain PyTorch; the sm_100a kernels in
``ops/csrc`` are tested against these in fp32.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ..core import sph


# ------------------------------------------------------------------ dense / elementwise
def linear(x, weight, bias=None, act=None):
    y = F.linear(x, weight, bias)
    if act == "silu":
        y = F.silu(y)
    return y


def layernorm_silu(x, weight, bias, eps):
    return F.silu(F.layer_norm(x, (x.shape[-1],), weight, bias, eps))


def so3_linear(x, weight, bias, lmax):
    """out[b, (l,m), o] = sum_i x[b, (l,m), i] W[l, o, i] (+ bias on l = 0)."""
    idx = torch.cat([torch.full((2 * l + 1,), l, dtype=torch.long, device=x.device) for l in range(lmax + 1)])
    w = weight.index_select(0, idx)
    out = torch.einsum("bmi,moi->bmo", x, w)
    out = torch.cat([out[:, :1] + bias.view(1, 1, -1), out[:, 1:]], dim=1)
    return out


def gate(gating_scalars, x, expand_index, lmax):
    """SiLU(x[:, 0]) and tanh(g)[expand_index] * x[:, 1:] (reference ``activation.py:57-77``)."""
    n, c = x.shape[0], x.shape[2]
    g = torch.tanh(gating_scalars).view(n, lmax, c).index_select(1, expand_index)
    return torch.cat([F.silu(x[:, :1]), x[:, 1:] * g], dim=1)


def rms_norm_sh(x, affine_weight, affine_bias, balance_degree_weight, eps, residual=None):
    """Equivariant RMS norm (reference ``layer_norm.py:290-338``); with ``residual`` it
    normalises ``x + residual`` and also returns that sum."""
    if residual is not None:
        s = x + residual
        return rms_norm_sh(s, affine_weight, affine_bias, balance_degree_weight, eps), s
    lmax = affine_weight.shape[0] - 1
    l0 = x[:, :1]
    l0 = l0 - l0.mean(dim=2, keepdim=True)
    feat = torch.cat([l0, x[:, 1:]], dim=1)
    norm = torch.einsum("nic,ia->nac", feat.pow(2), balance_degree_weight.to(x.dtype))
    norm = (norm.mean(dim=2, keepdim=True) + eps).pow(-0.5)
    idx = torch.cat([torch.full((2 * l + 1,), l, dtype=torch.long, device=x.device) for l in range(lmax + 1)])
    w = affine_weight.index_select(0, idx).unsqueeze(0)
    out = feat * (norm * w)
    out = torch.cat([out[:, :1] + affine_bias.view(1, 1, -1), out[:, 1:]], dim=1)
    return out


# ------------------------------------------------------------------ edge frame
def edge_rotation(vec_yzx, lmax, mmax, Js, mapping):
    """rot[e] (m-major rows x l-major cols): the rows |m| <= mmax of D(0, -beta, -alpha).

    D(0, -beta, -alpha) = J X(-beta) J X(-alpha) rotates the edge direction onto the polar
    axis (reference ``rotation.py:19-39, 86-99`` with gamma = 0).
    """
    alpha, beta = sph.edge_euler_angles(vec_yzx)
    zero = torch.zeros_like(alpha)
    D = sph.block_diag_wigner(lmax, zero, -beta, -alpha, [J.to(vec_yzx.dtype) for J in Js])
    return D.index_select(1, mapping.m_to_lm.to(D.device))


def gather_message(x_node, src_feats, dst, extra):
    parts = [src_feats, x_node.index_select(0, dst)]
    if extra is not None:
        parts.append(extra)
    return torch.cat(parts, dim=2)


def so2_conv(x, rad, weights, bias0, m_size, extra, cout):
    """Per-|m| GEMMs on the m-major message ``x`` [E, R, C] (reference ``so2_layers.py:139-214``).

    ``weights[0]`` is ``fc_m0.weight``; ``weights[m]`` the pair weight of |m| = m acting on
    the concatenated (+m, -m) rows.  ``rad`` (or None) multiplies the inputs; its layout is
    [m0 (l, c) | m1 (l, c) | ...], shared by the +m and -m rows.
    Returns (out [E, R, cout], gating scalars [E, extra] or None).
    """
    E, _, C = x.shape
    n0 = m_size[0]
    x0 = x[:, :n0].reshape(E, n0 * C)
    if rad is not None:
        x0 = x0 * rad[:, : n0 * C]
    y0 = F.linear(x0, weights[0], bias0)
    g = y0[:, :extra] if extra else None
    outs = [y0[:, extra:].reshape(E, n0, cout)]
    off, roff = n0, n0 * C
    for m in range(1, len(m_size)):
        k = m_size[m]
        xm = x[:, off : off + 2 * k].reshape(E, 2, k * C)
        if rad is not None:
            xm = xm * rad[:, roff : roff + k * C].unsqueeze(1)
        ym = F.linear(xm.reshape(E, 2 * k * C), weights[m])
        outs.append(ym.reshape(E, 2 * k, cout))
        off += 2 * k
        roff += k * C
    return torch.cat(outs, dim=1), g


def rotate_back(msg, rot):
    return torch.bmm(rot.transpose(1, 2), msg)


def scatter_sum(msg_l, dst, num_nodes):
    out = msg_l.new_zeros((num_nodes,) + tuple(msg_l.shape[1:]))
    return out.index_add_(0, dst, msg_l)


def edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge, src_feats=None):
    """One Edgewise message pass (reference ``esen_block.py:146-258``)."""
    c1, c2 = mod.so2_conv_1, mod.so2_conv_2
    rad = c1.rad_func(x_edge)
    if src_feats is None:
        src_feats = x_node.index_select(0, graph.src)
    msg = gather_message(x_node, src_feats, graph.dst, x_msg_edge)
    msg = torch.bmm(graph.rot, msg)
    h, g = so2_conv(msg, rad, c1.gemm_weights(), c1.fc_m0.bias, c1.m_size, c1.extra_m0_output_channels,
                    c1.m_output_channels)
    h = gate(g, h, mod.act.expand_index, mod.lmax)
    y, _ = so2_conv(h, None, c2.gemm_weights(), c2.fc_m0.bias, c2.m_size, 0, c2.m_output_channels)
    y = rotate_back(y, graph.rot)
    if node_or_edge == "node":
        return scatter_sum(y, graph.dst_out, graph.num_out)
    return y


def rotate_back_m0(e, rot):
    """Rotate m = 0 coefficients [E, L+1, C] back to the l-major frame [E, (L+1)^2, C]."""
    n0 = e.shape[1]
    return torch.bmm(rot[:, :n0].transpose(1, 2), e)


# ------------------------------------------------------------------ losses
def fock_loss(node_out, edge_out, node_target, edge_target, node_mask, edge_mask, loss_fn):
    """Masked node/edge/total loss as in ``splittrainer.py:1172-1233`` (closed shell)."""
    no = node_out[node_mask]
    eo = edge_out[edge_mask]
    nt = node_target[node_mask]
    et = edge_target[edge_mask]
    ln = loss_fn(no, nt)
    le = loss_fn(eo, et)
    lt = loss_fn(torch.cat([no, eo]), torch.cat([nt, et]))
    return ln, le, lt


# ------------------------------------------------------------------ heads
def fock_head_process(x, ws, bs, layer_params, act, act_scale, abs_gates):
    """Fock-head core on [N, (L+1)^2, C] (reference ``esen_osh.py:986-1052``).

    Scalars -> linear -> (C transformed scalars | L*C gates); gates -> (abs) -> act*scale;
    per-degree gated irreps -> per-degree linear.  Output is grouped by l with e3nn's
    (channel, m) flattening: [N, sum_l mul_out_l (2l+1)].
    """
    N, S, C = x.shape
    L = int(round(S ** 0.5)) - 1
    s = F.linear(x[:, 0], ws, bs)
    t0, g = s[:, :C], s[:, C:]
    if abs_gates:
        g = g.abs()
    g = (torch.sigmoid(g) if act == "sigmoid" else torch.tanh(g)) * act_scale
    g = g.view(N, L, C)
    outs = []
    for l in range(L + 1):
        w, b = layer_params[l]
        if w is None:
            continue
        xl = t0.unsqueeze(1) if l == 0 else x[:, l * l : (l + 1) ** 2] * g[:, l - 1].unsqueeze(1)
        yl = F.linear(xl, w, b)
        outs.append(yl.transpose(1, 2).reshape(N, -1))
    return torch.cat(outs, dim=1)


def gather_scale(x, idx, mult=None):
    """out[:, k] = x[:, idx[k]] * mult[k] (idx < 0 -> 0): one gather and one multiply by the
    combined column weights (validity times ``mult``)."""
    w = (idx >= 0).to(x.dtype)
    if mult is not None:
        w = w * mult.to(x.dtype)
    return x.index_select(1, idx.clamp(min=0)) * w
