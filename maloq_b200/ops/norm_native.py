"""Autograd wrappers of the norm / gate kernels and the per-degree (SO3) linear.

* :func:`rms_norm_sh` - equivariant RMS norm, optionally fused with the residual add;
* :func:`layernorm_silu` - silu(LayerNorm(x)) with a bf16 output (the next GEMM's operand);
* :func:`gate_l` - l-outer gate of the atomwise block;
* :func:`so3_linear` - per-degree channel mixing as tcgen05 GEMM problems, one per
  coefficient (strided views of the [B, S, C] layout, no copies), weight gradients as
  deterministic split-K GEMMs summed per degree.
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


def _partial_grid(rows):
    return max(1, min(int(rows), 148 * 4))


class _RmsNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, res, aw, ab, eps, out_dtype):
        lib = _lib()
        L = aw.shape[0] - 1
        x = x.contiguous().float()
        res_c = res.contiguous().float() if res is not None else None
        out = torch.empty(x.shape, device=x.device, dtype=out_dtype)
        s = torch.empty_like(x) if res is not None else None
        lib.rms_norm_fwd(L, x, res_c, aw.contiguous(), ab.contiguous(), out, s, eps)
        count_launches(1)
        ctx.save_for_backward(s if s is not None else x, aw)
        ctx.eps, ctx.has_res = eps, res is not None
        if res is not None:
            return out, s
        return out

    @staticmethod
    def backward(ctx, g_out, g_s=None):
        lib = _lib()
        s, aw = ctx.saved_tensors
        L = aw.shape[0] - 1
        B, S, C = s.shape
        grid = _partial_grid(B)
        dx = torch.empty_like(s)
        part = torch.empty(grid, L + 2, C, device=s.device, dtype=torch.float32)
        gs = g_s.contiguous().float() if (ctx.has_res and g_s is not None) else None
        if g_out is None:
            g_out = torch.zeros_like(s)
        g_out = g_out.contiguous()
        if g_out.dtype not in (torch.float32, torch.bfloat16):
            g_out = g_out.float()
        lib.rms_norm_bwd(L, s, g_out, gs, aw.contiguous(), dx, part, ctx.eps)
        count_launches(1)
        p = _colsum(part.view(part.shape[0], -1)).view(part.shape[1:])
        daw, dab = p[: L + 1], p[L + 1]
        if ctx.has_res:
            return dx, dx, daw, dab, None, None
        return dx, None, daw, dab, None, None


def rms_norm_sh(x, aw, ab, eps, residual=None, out_dtype=None):
    return _RmsNorm.apply(x, residual, aw, ab, eps, out_dtype or torch.float32)


class _LnSilu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous().float()
        out = torch.empty(x2.shape, device=x.device, dtype=torch.bfloat16)
        _lib().ln_silu_fwd(x2, w.contiguous(), b.contiguous(), out, eps)
        count_launches(1)
        ctx.save_for_backward(x2, w, b)
        ctx.eps, ctx.shape = eps, shape
        return out.view(shape)

    @staticmethod
    def backward(ctx, g):
        x2, w, b = ctx.saved_tensors
        M, W = x2.shape
        grid = max(1, min((M + 7) // 8, 148 * 4))
        dx = torch.empty_like(x2)
        part = torch.empty(grid * 8, 2, W, device=x2.device, dtype=torch.float32)
        _lib().ln_silu_bwd(x2, w.contiguous(), b.contiguous(), g.reshape(M, W).to(torch.bfloat16).contiguous(), dx,
                           part, ctx.eps)
        count_launches(1)
        p = _colsum(part.view(part.shape[0], -1)).view(part.shape[1:])
        return dx.view(ctx.shape), p[0], p[1], None


def layernorm_silu(x, w, b, eps=1e-5):
    return _LnSilu.apply(x, w, b, eps)


class _GateL(torch.autograd.Function):
    """fp32 or bf16 activations (output in the input's dtype); gates fp32.  ``silu_gates``: the
    gates are pre-activations whose SiLU the kernels apply (and differentiate) themselves."""

    @staticmethod
    def forward(ctx, gates, x, lmax, silu_gates):
        x = x.contiguous()
        if x.dtype != torch.bfloat16:
            x = x.float()
        gates = gates.contiguous().float()
        out = torch.empty_like(x)
        _lib().gate_l_fwd(lmax, x, gates, out, silu_gates)
        count_launches(1)
        ctx.save_for_backward(x, gates)
        ctx.lmax, ctx.silu_gates = lmax, silu_gates
        return out

    @staticmethod
    def backward(ctx, g):
        x, gates = ctx.saved_tensors
        dx = torch.empty_like(x)
        dg = torch.empty_like(gates)
        _lib().gate_l_bwd(ctx.lmax, x, gates, g.to(x.dtype).contiguous(), dx, dg, ctx.silu_gates)
        count_launches(1)
        return dg, dx, None, None


def gate_l(gates, x, lmax, silu_gates=False):
    return _GateL.apply(gates, x, lmax, silu_gates)


def _coef_l(S):
    out = []
    l = 0
    for j in range(S):
        while (l + 1) * (l + 1) <= j:
            l += 1
        out.append(l)
    return out


def _run_problems(As, Ws, Cs, biases, mn=False, splits=1, resids=None):
    lib = _lib()
    for i in range(0, len(As), 8):
        lib.gemm(As[i:i + 8], Ws[i:i + 8], Cs[i:i + 8], biases[i:i + 8], mn, 0, 1.0, splits, 128,
                 resids[i:i + 8] if resids is not None else [])
        count_launches(1)


class _SO3Linear(torch.autograd.Function):
    """out[:, j] = x[:, j] @ W[l_j]^T (+ bias on j = 0) (+ residual), one GEMM problem per
    coefficient j.  x fp32 or bf16 (cast once to bf16); output fp32 (with the residual added in
    the GEMM epilogue) or bf16; the input gradient comes back in the input's dtype.

    With a side weight ``sw`` [Ns, C] (and bias ``sb``) it also returns the scalar linear
    ``pre = x[:, 0] @ sw^T + sb`` (fp32) of the same input - the atomwise block's gate scalars -
    whose input gradient is added to row 0 of dx in place, instead of autograd building a
    full-size zero gradient for the row selection and adding it."""

    @staticmethod
    def forward(ctx, x, weight, bias, out_dtype, residual, sw=None, sb=None):
        B, S, C = x.shape
        Co = weight.shape[1]
        xb = x.to(torch.bfloat16).contiguous().view(B, S * C)
        wb = W.bf16(weight)
        out = torch.empty(B, S * Co, device=x.device, dtype=out_dtype)
        ls = _coef_l(S)
        res = None
        if residual is not None:
            res = residual.contiguous().float().view(B, S * Co)
        _run_problems([xb[:, j * C:(j + 1) * C] for j in range(S)], [wb[ls[j]] for j in range(S)],
                      [out[:, j * Co:(j + 1) * Co] for j in range(S)],
                      [bias.float().contiguous()] + [None] * (S - 1),
                      resids=None if res is None else [res[:, j * Co:(j + 1) * Co] for j in range(S)])
        ctx.dims = (B, S, C, Co)
        ctx.in_dtype = x.dtype
        ctx.has_res = residual is not None
        ctx.side = sw is not None
        ctx.has_sb = sb is not None
        if sw is None:
            ctx.save_for_backward(xb, weight)
            return out.view(B, S, Co)
        from .kernels import gemm_nt

        pre = gemm_nt(xb[:, :C], sw, sb, out_dtype=torch.float32, w_bf16=W.bf16(sw))
        ctx.save_for_backward(xb, weight, sw)
        return out.view(B, S, Co), pre

    @staticmethod
    def backward(ctx, g, g_pre=None):
        saved = ctx.saved_tensors
        xb, weight = saved[:2]
        B, S, C, Co = ctx.dims
        ls = _coef_l(S)
        L = ls[-1]
        gb = g.to(torch.bfloat16).contiguous().view(B, S * Co)
        dx_dtype = torch.bfloat16 if ctx.in_dtype == torch.bfloat16 else torch.float32
        dx = torch.empty(B, S * C, device=g.device, dtype=dx_dtype)
        wt = W.bf16_t(weight)
        _run_problems([gb[:, j * Co:(j + 1) * Co] for j in range(S)], [wt[ls[j]] for j in range(S)],
                      [dx[:, j * C:(j + 1) * C] for j in range(S)], [None] * S)
        splits = max(1, min(-(-296 // S), B // 2048, 16))
        part = torch.empty(S, splits, Co, C, device=g.device, dtype=torch.float32)
        _run_problems([gb[:, j * Co:(j + 1) * Co] for j in range(S)], [xb[:, j * C:(j + 1) * C] for j in range(S)],
                      [part[j] for j in range(S)], [None] * S, mn=True, splits=splits)
        dw = torch.empty(L + 1, Co, C, device=g.device, dtype=torch.float32)
        # each degree's sum over its coefficients and splits: row segments of part, one launch
        _lib().colsum_segments(part.view(S * splits, Co * C), [l * l * splits for l in range(L + 2)], dw)
        count_launches(1)
        db = _colsum(g[:, 0])
        dres = g if ctx.has_res else None
        dsw = dsb = None
        if ctx.side and g_pre is not None:
            from .kernels import gemm_nt, gemm_tn_weight_grad

            sw = saved[2]
            gp = g_pre.to(torch.bfloat16).contiguous()
            dx[:, :C] += gemm_nt(gp, sw, w_bf16=W.bf16_t(sw)).to(dx.dtype)
            dsw = gemm_tn_weight_grad(gp, xb[:, :C].contiguous())[: sw.shape[0], : sw.shape[1]]
            dsb = _colsum(g_pre) if ctx.has_sb else None
        return dx.view(B, S, C).to(ctx.in_dtype), dw, db, None, dres, dsw, dsb


def so3_linear(x, weight, bias, lmax, out_dtype=None, residual=None):
    return _SO3Linear.apply(x, weight, bias, out_dtype or torch.float32, residual)


def so3_linear_scalar(x, weight, bias, lmax, out_dtype, sw, sb):
    """(so3_linear(x), x[:, 0] @ sw^T + sb) with one autograd node (see ``_SO3Linear``)."""
    return _SO3Linear.apply(x, weight, bias, out_dtype or torch.float32, None, sw, sb)
