"""Coupled <-> uncoupled basis transform of label rows (block-diagonal CG matrix).

``apply_transform(x, W)`` = ``x @ W`` for the block-diagonal W of
:class:`maloq_b200.core.wigner3j.BasisTransform`; CUDA tensors run the block-sparse kernel
(only the non-zero CG blocks are multiplied).  Reference ``utils_tensor_decomp.py:154-169``.
"""

from __future__ import annotations

import torch

from . import _cuda, _native


def apply_transform(x, W):
    if _cuda(x):
        return _native.basis_transform(x, W)
    return torch.matmul(x, W)
