"""Op layer: every hot op of the model, with one CUDA implementation (sm_100a kernels in
``ops/csrc``) used for CUDA tensors and the PyTorch definition (``ops/reference.py``) used
for CPU tensors.  On a CUDA tensor an op whose kernel library is not built raises
instead of falling back.
"""

from __future__ import annotations

from . import reference as _ref
from . import native as _native

__all__ = [
    "edge_inputs", "embedding", "gemm_operand", "linear", "layernorm_silu", "so3_linear", "so3_linear_scalar", "gate", "gate_silu", "rms_norm_sh", "edge_rotation", "edgewise",
    "rotate_back_m0_scatter", "rotate_back_m0", "fock_loss",
]


_FORCE_TORCH = False


def launch_count() -> int:
    """Number of this library's CUDA kernels launched so far in this process."""
    return _native.launch_count()


def use_torch_ops(flag: bool = True) -> None:
    """Run the PyTorch definitions on CUDA tensors too (the NCCL/PyTorch baseline arm and
    the oracle side of kernel tests)."""
    global _FORCE_TORCH
    _FORCE_TORCH = bool(flag)


def _cuda(*tensors) -> bool:
    if _FORCE_TORCH:
        return False
    for t in tensors:
        if t is not None and hasattr(t, "is_cuda"):
            return bool(t.is_cuda)
    return False


def edge_inputs(src_z, dst_z, edge_attr, src_weight, dst_weight, offset, coeff):
    """Radial-MLP input rows [src_weight[src_z] | exp(coeff (d - offset)^2) | dst_weight[dst_z]]
    with d = edge_attr[:, 0]: one kernel writing the bf16 GEMM operand on the kernel path."""
    if _cuda(src_weight):
        return _native.edge_inputs(src_z, dst_z, edge_attr, src_weight, dst_weight, offset, coeff)
    import torch

    g = torch.exp(coeff * (edge_attr[:, 0].view(-1, 1) - offset.view(1, -1)) ** 2)
    return torch.cat([src_weight.index_select(0, src_z), g, dst_weight.index_select(0, dst_z)], dim=1)


def embedding(idx, weight):
    """weight[idx] (an ``nn.Embedding`` lookup); on the kernel path its backward needs no
    host synchronisation."""
    if _cuda(weight):
        return _native.embedding(idx, weight)
    return weight.index_select(0, idx)


def gemm_operand(x):
    """``x`` in the dtype the kernel path's GEMMs read (bf16) when it only feeds GEMMs - cast once
    instead of once per consumer, with its gradient accumulated in that dtype too; unchanged on
    the PyTorch path."""
    if _cuda(x):
        import torch

        return x.to(torch.bfloat16)
    return x


def linear(x, weight, bias=None, act=None, out_dtype=None):
    """x @ weight^T + bias (optional SiLU).  ``out_dtype`` (CUDA path): dtype of the result,
    e.g. bf16 when the next consumer reads bf16 (fp32 by default)."""
    if _cuda(x):
        return _native.linear(x, weight, bias, act, out_dtype)
    return _ref.linear(x, weight, bias, act)


def layernorm_silu(x, weight, bias, eps=1e-5):
    if _cuda(x):
        return _native.layernorm_silu(x, weight, bias, eps)
    return _ref.layernorm_silu(x, weight, bias, eps)


def so3_linear(x, weight, bias, lmax, out_dtype=None, residual=None):
    """Per-degree linear; ``residual`` (same shape as the output, fp32) is added to the result
    (fused into the GEMM epilogue on the kernel path); ``out_dtype`` selects a bf16 output on
    the kernel path."""
    if _cuda(x):
        return _native.so3_linear(x, weight, bias, lmax, out_dtype, residual)
    out = _ref.so3_linear(x.to(weight.dtype), weight, bias, lmax)
    return out if residual is None else out + residual


def so3_linear_scalar(x, weight, bias, lmax, out_dtype, scalar_weight, scalar_bias):
    """(so3_linear(x), x[:, 0] @ scalar_weight^T + scalar_bias): the atomwise block's SO3 linear
    and the linear of its gate scalars, which read the same input (one autograd node on the
    kernel path, so the scalar linear's input gradient is added into row 0 in place)."""
    if _cuda(x):
        return _native.so3_linear_scalar(x, weight, bias, lmax, out_dtype, scalar_weight, scalar_bias)
    return _ref.so3_linear(x.to(weight.dtype), weight, bias, lmax), _ref.linear(x[:, 0].to(weight.dtype),
                                                                                 scalar_weight, scalar_bias)


def gate(gating_scalars, x, expand_index, lmax):
    if _cuda(x):
        return _native.gate(gating_scalars, x, expand_index, lmax)
    return _ref.gate(gating_scalars, x, expand_index, lmax)


def gate_silu(pre, x, expand_index, lmax):
    """``gate(silu(pre), x, ...)`` with the SiLU inside the gate kernels on the kernel path (no
    separate pass over the gate pre-activations in forward or backward)."""
    if _cuda(x):
        return _native.gate_silu(pre, x, expand_index, lmax)
    import torch

    return _ref.gate(torch.nn.functional.silu(pre), x, expand_index, lmax)


def rms_norm_sh(x, affine_weight, affine_bias, balance_degree_weight, eps, residual=None, out_dtype=None):
    """``out_dtype``: dtype of the normalised output on the kernel path (bf16 when it only
    feeds a GEMM); the residual sum stays fp32."""
    if _cuda(x):
        return _native.rms_norm_sh(x, affine_weight, affine_bias, eps, residual, out_dtype)
    return _ref.rms_norm_sh(x, affine_weight, affine_bias, balance_degree_weight, eps, residual)


def edge_rotation(vec_yzx, lmax, mmax, Js, mapping):
    if _cuda(vec_yzx):
        return _native.edge_rotation(vec_yzx, lmax, mmax, Js, mapping)
    return _ref.edge_rotation(vec_yzx, lmax, mmax, Js, mapping)


def _src_feats(x_node, graph):
    if graph.halo is not None:
        return graph.halo.gather_source(x_node, graph)
    return None


def edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge):
    if _cuda(x_node):
        return _native.edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge)
    return _ref.edgewise(mod, x_node, x_msg_edge, x_edge, graph, node_or_edge, _src_feats(x_node, graph))


def rotate_back_m0_scatter(e, graph, x_node, scale):
    if _cuda(e):
        return _native.rotate_back_m0_scatter(e, graph, x_node, scale)
    y = _ref.rotate_back_m0(e, graph.rot)
    return x_node + _ref.scatter_sum(y * scale, graph.dst_out, graph.num_out).to(x_node.dtype)


def rotate_back_m0(e, graph):
    if _cuda(e):
        return _native.rotate_back_m0(e, graph)
    return _ref.rotate_back_m0(e, graph.rot)


def fock_loss(node_out, edge_out, node_target, edge_target, node_mask, edge_mask, loss_fn):
    return _ref.fock_loss(node_out, edge_out, node_target, edge_target, node_mask, edge_mask, loss_fn)


def fock_head_process(x, ws, bs, layer_params, act, act_scale, abs_gates):
    if _cuda(x):
        return _native.fock_head_process(x, ws, bs, layer_params, act, act_scale, abs_gates)
    return _ref.fock_head_process(x, ws, bs, layer_params, act, act_scale, abs_gates)


def gather_scale(x, idx, mult=None):
    if _cuda(x):
        return _native.gather_scale(x, idx, mult)
    return _ref.gather_scale(x, idx, mult)
