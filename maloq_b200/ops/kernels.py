"""Kernel-backed implementations of the op layer (registered into :mod:`.native`).

Every function here runs sm_100a kernels from the in-tree library (``ops/_ext.py``).
GEMM-shaped work goes to the tcgen05 GEMM; operands are bf16 with fp32 accumulation and
fp32 master weights (weights are cast to bf16 per call; gradients come back in fp32).
"""

from __future__ import annotations

import torch

from . import _ext
from . import reference as _ref
from . import weights as W
from .native import count_launches, register

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _ext.load()
    return _lib


def error_status(clear=True) -> int:
    return int(lib().error_status(clear))


class DeviceError(RuntimeError):
    """A kernel of this library recorded an error code in the device error word."""


class CommTimeoutError(DeviceError):
    """A bounded device wait ran out: a peer GPU did not raise its flag (peer barrier, halo,
    fused all-reduce), or a GEMM pipeline stage never arrived."""


class BoundsError(DeviceError):
    """An index-checked build (``MALOQ_BOUNDS_CHECK=1``) found an out-of-range index and
    skipped the access."""


ERROR_CODES = {1: ("GEMM producer waited for a free stage", CommTimeoutError),
               2: ("GEMM MMA warp waited for operand tiles", CommTimeoutError),
               3: ("GEMM epilogue waited for the accumulator", CommTimeoutError),
               4: ("a peer GPU did not arrive at a peer barrier", CommTimeoutError),
               5: ("an index was out of range", BoundsError)}


def check_device_status(where="") -> None:
    """Read and clear the device error word; raise the matching :class:`DeviceError` if a
    kernel recorded one (the read synchronises the device)."""
    code = error_status(clear=True)
    if code == 0:
        return
    if code < 0:
        raise DeviceError(f"could not read the device error word{' after ' + where if where else ''}")
    msg, cls = ERROR_CODES.get(code, (f"unknown error code {code}", DeviceError))
    raise cls(f"device error {code}: {msg}{' (after ' + where + ')' if where else ''}")


# ------------------------------------------------------------------ GEMM helpers
def _pad_cols(t, mult=8):
    k = t.shape[-1]
    if k % mult == 0:
        return t
    return torch.nn.functional.pad(t, (0, mult - k % mult))


def gemm_nt(a, w, bias=None, out_dtype=torch.float32, act=0, alpha=1.0, bn=None, w_bf16=None):
    """out[M,N] = alpha * a[M,K] @ w[N,K]^T (+bias) (silu if act); bf16 operands.  ``w_bf16``:
    a ready bf16 copy of ``w`` (the weight cache)."""
    a = _pad_cols(a.to(torch.bfloat16)).contiguous()
    w = _pad_cols(w_bf16 if w_bf16 is not None else w.to(torch.bfloat16))
    N = w.shape[0]
    if N % 8:
        w = torch.nn.functional.pad(w, (0, 0, 0, 8 - N % 8))
        if bias is not None:
            bias = torch.nn.functional.pad(bias, (0, 8 - N % 8))
    w = w.contiguous()
    out = torch.empty(a.shape[0], w.shape[0], device=a.device, dtype=out_dtype)
    if a.shape[0] > 0:
        lib().gemm([a], [w], [out], [None if bias is None else bias.float().contiguous()], False, act, alpha, 1,
                   bn or (128 if w.shape[0] <= 128 else 256))
        count_launches(1)
    return out[:, :N] if out.shape[1] != N else out


def colsum(x):
    """fp32 [N] column sums of a 2-D fp32/bf16 tensor in a fixed order (bias gradients and
    per-CTA partial sums); any row stride, unit column stride."""
    if x.dim() != 2 or (x.shape[1] > 1 and x.stride(1) != 1) or x.dtype not in (torch.float32, torch.bfloat16):
        x = x.reshape(-1, x.shape[-1]).float().contiguous()
    out = torch.empty(x.shape[1], device=x.device, dtype=torch.float32)
    lib().colsum(x, out)
    count_launches(1 if x.shape[0] <= 4096 else 2)
    return out


def gemm_tn_weight_grad(gy, x):
    """dW[N,K] = gy[M,N]^T @ x[M,K] with deterministic split-K over M (fp32 result)."""
    gy = _pad_cols(gy.to(torch.bfloat16)).contiguous()
    x = _pad_cols(x.to(torch.bfloat16)).contiguous()
    M, N = gy.shape
    K = x.shape[1]
    out = torch.empty(N, K, device=gy.device, dtype=torch.float32)
    if M == 0:
        return out.zero_()
    bn = 128
    tiles = ((N + 127) // 128) * ((K + bn - 1) // bn)
    splits = max(1, min(-(-296 // tiles), M // 1024, 64))
    if splits == 1:
        lib().gemm([gy], [x], [out], [None], True, 0, 1.0, 1, bn)
        count_launches(1)
    else:
        part = torch.empty(splits, N, K, device=gy.device, dtype=torch.float32)
        lib().gemm([gy], [x], [part], [None], True, 0, 1.0, splits, bn)
        lib().splitk_reduce(part, out, 0.0)
        count_launches(2)
    return out


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, out_dtype):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        y = gemm_nt(x2, weight, bias, out_dtype=out_dtype, w_bf16=W.bf16(weight))
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.in_shape, ctx.in_dtype = shape, x.dtype
        return y.reshape(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, weight = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1]).to(torch.bfloat16).contiguous()
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = gemm_nt(g2, weight, w_bf16=W.bf16_t(weight)).to(ctx.in_dtype).reshape(ctx.in_shape)
        if ctx.needs_input_grad[1]:
            gw = gemm_tn_weight_grad(g2, x2)[: weight.shape[0], : weight.shape[1]]
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = colsum(gy.reshape(-1, gy.shape[-1]))
        return gx, gw, gb, None


class _Embedding(torch.autograd.Function):
    """Embedding rows with a backward that needs no device-to-host read: the weight gradient is
    one_hot(idx)^T @ g, one dense GEMM (deterministic), instead of the sort-and-segment
    reduction of the stock backward, which reads a segment count back to the host for large
    index counts (one synchronisation per call)."""

    @staticmethod
    def forward(ctx, idx, weight):
        ctx.save_for_backward(idx)
        ctx.n_rows = weight.shape[0]
        return weight.index_select(0, idx)

    @staticmethod
    def backward(ctx, g):
        (idx,) = ctx.saved_tensors
        onehot = (idx.unsqueeze(1) == torch.arange(ctx.n_rows, device=idx.device)).to(g.dtype)
        return None, onehot.t() @ g


@register("edge_inputs")
def edge_inputs(src_z, dst_z, edge_attr, src_w, dst_w, offset, coeff):
    from . import misc_native

    return misc_native.edge_inputs(src_z, dst_z, edge_attr, src_w, dst_w, offset, coeff)


@register("embedding")
def embedding(idx, weight):
    return _Embedding.apply(idx, weight)


@register("linear")
def linear(x, weight, bias=None, act=None, out_dtype=None):
    y = _Linear.apply(x, weight, bias, out_dtype or torch.float32)
    if act == "silu":
        y = torch.nn.functional.silu(y)
    return y


# ------------------------------------------------------------------ ops still on PyTorch glue
# These run PyTorch on the CUDA tensors until their fused kernels land; each is listed so the
# set of non-kernel ops is explicit.
TORCH_GLUE = ("gather_scale",)


@register("layernorm_silu")
def layernorm_silu(x, w, b, eps):
    from . import norm_native

    return norm_native.layernorm_silu(x, w, b, eps)


@register("gate")
def gate(gating_scalars, x, expand_index, lmax):
    from . import norm_native

    return norm_native.gate_l(gating_scalars, x, lmax)


@register("gate_silu")
def gate_silu(pre, x, expand_index, lmax):
    from . import norm_native

    return norm_native.gate_l(pre, x, lmax, silu_gates=True)


@register("rms_norm_sh")
def rms_norm_sh(x, aw, ab, eps, residual=None, out_dtype=None):
    from . import norm_native

    return norm_native.rms_norm_sh(x, aw, ab, eps, residual, out_dtype)


register("gather_scale")(_ref.gather_scale)
register("fock_head_process")(lambda x, ws, bs, lp, act, sc, ab: _head_process(x, ws, bs, lp, act, sc, ab))
from . import labels_native  # noqa: E402

for _name in ("basis_transform", "matrix_to_labels", "labels_to_matrix", "blocks_to_coupled", "coupled_to_blocks"):
    register(_name)(getattr(labels_native, _name))


@register("so3_linear")
def so3_linear(x, weight, bias, lmax, out_dtype=None, residual=None):
    from . import norm_native

    return norm_native.so3_linear(x, weight, bias, lmax, out_dtype, residual)


@register("so3_linear_scalar")
def so3_linear_scalar(x, weight, bias, lmax, out_dtype, sw, sb):
    from . import norm_native

    return norm_native.so3_linear_scalar(x, weight, bias, lmax, out_dtype, sw, sb)


def _pad8(n):
    return (n + 7) // 8 * 8


_HEAD_COLS = {}


class _FockHeadFn(torch.autograd.Function):
    """Gated per-degree projections of the Fock head (reference ``esen_osh.py:986-1052``).

    ``head_gate`` writes the bf16 GEMM operand A [N, S, C] in one pass (row 0 the transformed
    scalars, every l >= 1 coefficient times its activated gate).  One grouped-GEMM problem per
    coefficient j projects A[:, j] with its degree's weight into column block j of one fp32
    buffer Y (blocks padded to 8 columns); one gather puts Y's columns into the head's sorted
    order (per degree, e3nn's (channel, m) flattening).  The scalar linear (x[:, 0] ->
    transformed scalars | raw gates) runs inside, so its input gradient lands in row 0 of dx
    directly (no full-size zero gradient for the row selection).  Backward: the gather's
    transpose, one grouped input-gradient GEMM, split-K weight gradients summed per degree in a
    fixed order, ``head_gate_bwd`` for the gradients of x and of the scalar linear's output, and
    the scalar linear's gradients."""

    @staticmethod
    def forward(ctx, x, ws_s, bs_s, act, scale, absg, present, *wb):
        from .norm_native import _run_problems

        N, S, C = x.shape
        x0 = x[:, 0].to(torch.bfloat16).contiguous()
        sv = gemm_nt(x0, ws_s, bs_s, out_dtype=torch.float32, w_bf16=W.bf16(ws_s))
        L = int(round(S ** 0.5)) - 1
        ls = [l for l in range(L + 1) if present[l]]
        ws = dict(zip(ls, wb[0::2]))
        bs = dict(zip(ls, wb[1::2]))
        mul = {l: ws[l].shape[0] for l in ls}
        x = x.contiguous().float()
        sv = sv.contiguous().float()
        A = torch.empty(N, S, C, device=x.device, dtype=torch.bfloat16)
        lib().head_gate_fwd(L, x, sv, A, 0 if act == "sigmoid" else 1, float(scale), bool(absg))
        js = [j for j in range(S) if int(j ** 0.5) in mul]
        lj = {j: int(j ** 0.5) for j in js}
        off, o = {}, 0
        for j in js:
            off[j] = o
            o += _pad8(mul[lj[j]])
        key = (x.device, L, tuple(sorted(mul.items())))
        if key not in _HEAD_COLS:
            cols = [off[l * l + m] + oo for l in ls for oo in range(mul[l]) for m in range(2 * l + 1)]
            _HEAD_COLS[key] = torch.tensor(cols, dtype=torch.long, device=x.device)
        cols = _HEAD_COLS[key]
        wpad, bpad = {}, {}
        for l in ls:
            w = ws[l].to(torch.bfloat16)
            wpad[l] = torch.nn.functional.pad(w, (0, 0, 0, _pad8(mul[l]) - mul[l])).contiguous()
            bpad[l] = None if bs[l] is None else \
                torch.nn.functional.pad(bs[l].float(), (0, _pad8(mul[l]) - mul[l])).contiguous()
        Y = torch.empty(N, o, device=x.device, dtype=torch.float32)
        A2 = A.view(N, S * C)
        if N > 0:
            _run_problems([A2[:, j * C:(j + 1) * C] for j in js], [wpad[lj[j]] for j in js],
                          [Y[:, off[j]:off[j] + _pad8(mul[lj[j]])] for j in js], [bpad[lj[j]] for j in js])
        count_launches(2)
        ctx.save_for_backward(x, sv, A, x0, ws_s, *[ws[l] for l in ls])
        ctx.meta = (L, ls, mul, js, lj, off, o, act, float(scale), bool(absg), cols, [bs[l] is not None for l in ls],
                    bs_s is not None)
        return Y.index_select(1, cols)

    @staticmethod
    def backward(ctx, g):
        from .norm_native import _run_problems

        saved = ctx.saved_tensors  # read once (a second read fails under non-reentrant checkpointing)
        x, sv, A, x0, ws_s = saved[:5]
        wlist = saved[5:]
        L, ls, mul, js, lj, off, width, act, scale, absg, cols, has_b, has_bs = ctx.meta
        N, S, C = x.shape
        dY = torch.zeros(N, width, device=g.device, dtype=torch.float32)
        dY.index_copy_(1, cols, g.float().contiguous())
        dYb = dY.to(torch.bfloat16)
        dA = torch.empty(N, S, C, device=g.device, dtype=torch.float32)
        dA2 = dA.view(N, S * C)
        for j in range(S):  # coefficients of degrees without outputs: no gradient reaches them
            if j not in lj:
                dA2[:, j * C:(j + 1) * C].zero_()
        wt = {l: torch.nn.functional.pad(w.to(torch.bfloat16), (0, 0, 0, _pad8(mul[l]) - mul[l])).t().contiguous()
              for l, w in zip(ls, wlist)}
        splits = max(1, min(-(-296 // max(1, len(js))), N // 2048, 16))
        # split-K partials of the weight gradients, one contiguous block per degree so that each
        # degree's gradient is a single reduction over (coefficient, split)
        partsL = {l: torch.empty(2 * l + 1, splits, _pad8(mul[l]), C, device=g.device, dtype=torch.float32)
                  for l in ls}
        parts = {j: partsL[lj[j]][j - lj[j] ** 2] for j in js}
        A2 = A.view(N, S * C)
        if N > 0:
            _run_problems([dYb[:, off[j]:off[j] + _pad8(mul[lj[j]])] for j in js], [wt[lj[j]] for j in js],
                          [dA2[:, j * C:(j + 1) * C] for j in js], [None] * len(js))
            _run_problems([dYb[:, off[j]:off[j] + _pad8(mul[lj[j]])] for j in js],
                          [A2[:, j * C:(j + 1) * C] for j in js], [parts[j] for j in js], [None] * len(js),
                          mn=True, splits=splits)
        grads = []
        for l, hb in zip(ls, has_b):
            P, o0 = _pad8(mul[l]), off[l * l]
            pl = partsL[l]
            dw = colsum(pl.view(-1, P * C)).view(P, C) if N > 0 else torch.zeros(P, C, device=g.device)
            grads.append(dw[:mul[l]])
            # the degree's column blocks are adjacent in dY: [N, 2l+1, P]
            db = colsum(colsum(dY[:, o0:o0 + (2 * l + 1) * P]).view(2 * l + 1, P))[:mul[l]] if hb else None
            grads.append(db)
        dx = torch.empty_like(x)
        dsv = torch.empty_like(sv)
        lib().head_gate_bwd(L, x, sv, dA, dx, dsv, 0 if act == "sigmoid" else 1, scale, absg)
        count_launches(4)
        # the scalar linear: its input gradient is row 0 of dx (head_gate_bwd left it zero)
        d2 = dsv.to(torch.bfloat16)
        dx[:, 0] = gemm_nt(d2, ws_s, w_bf16=W.bf16_t(ws_s))
        dws = gemm_tn_weight_grad(d2, x0)[: ws_s.shape[0], : ws_s.shape[1]] if ctx.needs_input_grad[1] else None
        dbs = colsum(dsv) if has_bs and ctx.needs_input_grad[2] else None
        return (dx, dws, dbs, None, None, None, None, *grads)


def _head_process(x, ws, bs, layer_params, act, act_scale, abs_gates):
    present = tuple(w is not None for w, _ in layer_params)
    wb = []
    for w, b in layer_params:
        if w is not None:
            wb += [w, b]
    return _FockHeadFn.apply(x, ws, bs, act, act_scale, abs_gates, present, *wb)


@register("edgewise")
def edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge):
    from . import edge_native

    return edge_native.edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge)


def _so2_conv(x, rad, weights, bias0, m_size, extra, cout):
    E, _, C = x.shape
    n0 = m_size[0]
    x0 = x[:, :n0].reshape(E, n0 * C)
    if rad is not None:
        x0 = x0 * rad[:, : n0 * C]
    y0 = linear(x0, weights[0], bias0)
    g = y0[:, :extra] if extra else None
    outs = [y0[:, extra:].reshape(E, n0, cout)]
    off, roff = n0, n0 * C
    for m in range(1, len(m_size)):
        k = m_size[m]
        xm = x[:, off: off + 2 * k].reshape(E, 2, k * C)
        if rad is not None:
            xm = xm * rad[:, roff: roff + k * C].unsqueeze(1)
        ym = linear(xm.reshape(E, 2 * k * C), weights[m])
        outs.append(ym.reshape(E, 2 * k, cout))
        off += 2 * k
        roff += k * C
    return torch.cat(outs, dim=1), g


@register("rotate_back_m0")
def rotate_back_m0(e, graph):
    from . import edge_native

    return edge_native.rotate_back_m0(e, graph)


@register("rotate_back_m0_scatter")
def rotate_back_m0_scatter(e, graph, x_node, scale):
    from . import edge_native

    return edge_native.rotate_back_m0(e, graph, base=x_node, scale=scale)


@register("fock_loss")
def fock_loss(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt, name):
    from . import misc_native

    return misc_native.fock_loss(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt, name)


@register("edge_rotation")
def edge_rotation(vec_yzx, lmax, mmax, Js, mapping):
    from . import misc_native

    return misc_native.edge_rotation(vec_yzx, lmax, mmax, Js, mapping)

