"""Block-sparse Hamiltonian <-> label rows, and the fused label <-> coupled transform.

CUDA tensors run the kernels of ``ops/csrc/labels.cu``; CPU tensors the gathers below.
Reference: ``fock_utils/matrix2labels_kernels.py`` (K8-K12).
"""

from __future__ import annotations

import torch

from . import _cuda, _native


def _ref_m2l(data, block_ptr, pair_type, pos_table):
    pos = pos_table.index_select(0, pair_type)  # [B, D]
    valid = pos >= 0
    flat = block_ptr[:-1].unsqueeze(1) + pos.clamp(min=0)
    out = data[flat.reshape(-1)].reshape(pos.shape)
    return torch.where(valid, out, torch.zeros((), dtype=data.dtype, device=data.device))


def _ref_l2m(labels, block_ptr, pair_type, pos_table, n_data):
    pos = pos_table.index_select(0, pair_type)
    valid = pos >= 0
    flat = (block_ptr[:-1].unsqueeze(1) + pos.clamp(min=0))[valid]
    out = labels.new_zeros(n_data)
    out[flat] = labels[valid]
    return out


def matrix_to_labels(data, block_ptr, pair_type, pos_table):
    if _cuda(data):
        return _native.matrix_to_labels(data, block_ptr, pair_type, pos_table)
    return _ref_m2l(data, block_ptr, pair_type, pos_table)


def labels_to_matrix(labels, block_ptr, pair_type, pos_table, n_data):
    if _cuda(labels):
        return _native.labels_to_matrix(labels, block_ptr, pair_type, pos_table, n_data)
    return _ref_l2m(labels, block_ptr, pair_type, pos_table, n_data)


def blocks_to_coupled(data, block_ptr, pair_type, pos_table, transform):
    """Coupled label rows of block-sparse data: ``get_net_out(matrix_to_labels(...))`` in one
    pass on CUDA (gather + block-diagonal transform, ``ops/csrc/labels.cu``)."""
    if _cuda(data):
        return _native.blocks_to_coupled(data, block_ptr, pair_type, pos_table, transform)
    return transform.get_net_out(_ref_m2l(data, block_ptr, pair_type, pos_table))


def coupled_to_blocks(coupled, block_ptr, pair_type, pos_table, transform, n_data, out=None):
    """Block-sparse data of coupled label rows: ``labels_to_matrix(get_H(...))`` in one pass on
    CUDA (block-diagonal transform + scatter).  ``block_ptr[r]`` is row r's data offset; with
    ``out`` the rows' blocks are written into that buffer (other entries untouched)."""
    if _cuda(coupled):
        return _native.coupled_to_blocks(coupled, block_ptr, pair_type, pos_table, transform, n_data, out)
    unc = transform.get_H(coupled)
    if out is None:
        return _ref_l2m(unc, block_ptr, pair_type, pos_table, n_data)
    pos = pos_table.index_select(0, pair_type)
    valid = pos >= 0
    flat = (block_ptr[: pos.shape[0]].unsqueeze(1) + pos.clamp(min=0))[valid]
    out[flat] = unc[valid].to(out.dtype)
    return out
