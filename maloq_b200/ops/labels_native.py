"""CUDA side of the label ops: one row kernel (``basis_rows`` in ``ops/csrc/labels.cu``) does
block-sparse gather / dense rows -> block-diagonal transform -> scatter / dense rows.

* ``basis_transform`` - dense rows through the CG blocks (``get_H`` / ``get_net_out``);
* ``matrix_to_labels`` / ``labels_to_matrix`` - the identity transform with gather / scatter;
* ``blocks_to_coupled`` / ``coupled_to_blocks`` - gather or scatter fused with the transform.
Reference kernels: ``fock_utils/matrix2labels_kernels.py:689-800`` (block-sparse copies) and
``fock_utils/basis_transform_triton_backend.py:33-154`` (CG block GEMMs).
"""

from __future__ import annotations

import torch

from .native import count_launches


def _lib():
    from .kernels import lib

    return lib()


_IDENTITY = {}
_POS32 = {}


def _tables(transform, inverse, device, dtype, transpose=False):
    cache = transform.__dict__.setdefault("_device_tables", {})
    key = (bool(inverse), bool(transpose), str(device), dtype)
    if key not in cache:
        meta, coef = transform.column_tables(inverse, transpose)
        cache[key] = (torch.as_tensor(meta, device=device), torch.as_tensor(coef, device=device, dtype=dtype))
    return cache[key]


def _identity(d, device, dtype):
    key = (d, str(device), dtype)
    if key not in _IDENTITY:
        u = torch.arange(d, dtype=torch.int32)
        meta = torch.stack([u, torch.ones_like(u), u, torch.zeros_like(u)], 1).contiguous().to(device)
        _IDENTITY[key] = (meta, torch.ones(d, device=device, dtype=dtype))
    return _IDENTITY[key]


def _pos32(pos):
    key = (pos.data_ptr(), pos.shape, str(pos.device))
    hit = _POS32.get(key)
    if hit is None or hit[0] is not pos:
        hit = (pos, pos.to(torch.int32).contiguous())
        _POS32[key] = hit
    return hit[1]


def _dtype(x):
    return torch.float64 if x.dtype == torch.float64 else torch.float32


def _rows_transform(x, transform, inverse, transpose):
    dt = _dtype(x)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).to(dt).contiguous()
    meta, coef = _tables(transform, inverse, x.device, dt, transpose)
    out = torch.empty(x2.shape[0], meta.shape[0], device=x.device, dtype=dt)
    _lib().basis_rows(x2, out, None, None, None, meta, coef, x2.shape[1], x2.shape[0], False, False)
    count_launches(1)
    return out.reshape(*shape[:-1], meta.shape[0]).to(x.dtype)


class _BasisTransformFn(torch.autograd.Function):
    """x @ W (block diagonal); backward g @ W^T with the transposed tables."""

    @staticmethod
    def forward(ctx, x, transform, inverse):
        ctx.transform, ctx.inverse = transform, inverse
        return _rows_transform(x, transform, inverse, False)

    @staticmethod
    def backward(ctx, g):
        return _rows_transform(g.contiguous(), ctx.transform, ctx.inverse, True), None, None


def basis_transform(x, transform, inverse=False):
    if torch.is_grad_enabled() and x.requires_grad:
        return _BasisTransformFn.apply(x, transform, inverse)
    return _rows_transform(x, transform, inverse, False)


def _rows(ptr, pt):
    return ptr.contiguous(), pt.to(torch.long).contiguous()


def matrix_to_labels(data, block_ptr, pair_type, pos_table):
    dt = _dtype(data)
    D = pos_table.shape[1]
    meta, coef = _identity(D, data.device, dt)
    ptr, pt = _rows(block_ptr, pair_type)
    rows = pt.numel()
    out = torch.empty(rows, D, device=data.device, dtype=dt)
    _lib().basis_rows(data.to(dt).contiguous(), out, ptr, pt, _pos32(pos_table), meta, coef, D, rows, True, False)
    count_launches(1)
    return out.to(data.dtype)


def labels_to_matrix(labels, block_ptr, pair_type, pos_table, n_data):
    dt = _dtype(labels)
    D = pos_table.shape[1]
    meta, coef = _identity(D, labels.device, dt)
    ptr, pt = _rows(block_ptr, pair_type)
    rows = pt.numel()
    out = torch.zeros(int(n_data), device=labels.device, dtype=dt)
    _lib().basis_rows(labels.to(dt).contiguous(), out, ptr, pt, _pos32(pos_table), meta, coef, D, rows, False, True)
    count_launches(1)
    return out.to(labels.dtype)


def blocks_to_coupled(data, block_ptr, pair_type, pos_table, transform):
    dt = _dtype(data)
    meta, coef = _tables(transform, True, data.device, dt)
    ptr, pt = _rows(block_ptr, pair_type)
    rows = pt.numel()
    out = torch.empty(rows, meta.shape[0], device=data.device, dtype=dt)
    _lib().basis_rows(data.to(dt).contiguous(), out, ptr, pt, _pos32(pos_table), meta, coef, pos_table.shape[1], rows,
                      True, False)
    count_launches(1)
    return out.to(data.dtype)


def coupled_to_blocks(coupled, block_ptr, pair_type, pos_table, transform, n_data, out=None):
    dt = _dtype(coupled)
    meta, coef = _tables(transform, False, coupled.device, dt)
    ptr, pt = _rows(block_ptr, pair_type)
    rows = pt.numel()
    if out is not None:
        if out.dtype != dt or not out.is_contiguous():
            raise ValueError("coupled_to_blocks: out must be a contiguous buffer of the label dtype")
        _lib().basis_rows(coupled.to(dt).contiguous(), out, ptr, pt, _pos32(pos_table), meta, coef,
                          coupled.shape[1], rows, False, True)
        count_launches(1)
        return out
    out = torch.zeros(int(n_data), device=coupled.device, dtype=dt)
    _lib().basis_rows(coupled.to(dt).contiguous(), out, ptr, pt, _pos32(pos_table), meta, coef, coupled.shape[1], rows,
                      False, True)
    count_launches(1)
    return out.to(coupled.dtype)
