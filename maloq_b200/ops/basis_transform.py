"""Coupled <-> uncoupled basis transform of label rows (block-diagonal CG matrix).

``apply_transform(x, transform, inverse)`` = ``x @ W`` (``get_H``) or ``x @ W_inv``
(``get_net_out``) for a :class:`maloq_b200.core.wigner3j.BasisTransform`.  CUDA tensors run
the block-diagonal row kernel (``ops/csrc/labels.cu``: only the CG blocks are multiplied, at
the input precision); CPU tensors the dense matmul.  Reference
``fock_utils/utils_tensor_decomp.py:154-169``.
"""

from __future__ import annotations

import torch

from . import _cuda, _native


def apply_transform(x, transform, inverse=False):
    if _cuda(x):
        return _native.basis_transform(x, transform, inverse)
    W = transform.W_global_inv if inverse else transform.W_global
    return torch.matmul(x, W.to(x.device, x.dtype))
