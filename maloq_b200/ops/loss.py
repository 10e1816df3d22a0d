"""Masked Fock loss (node, edge and combined terms) - reference ``splittrainer.py:1172-1233``.

The padding mask of a label row is ``mask_table[pair_type]``.  For losses that are functions
of the masked sums of squared and absolute errors (``mse``/``rmse``/``rmse_mse``/``l1``/
``combined`` padded losses) CUDA tensors use one fused kernel that reduces the sums for
node and edge rows and, in backward, writes d(loss)/d(output) in a second pass; other loss
functions run the PyTorch definition.
"""

from __future__ import annotations

import torch

from . import _cuda, _native
from . import reference as _ref

# loss name -> (uses_sq, uses_abs, f(mse, mae) as torch expression)
DECOMPOSABLE = {
    "mse_padded_loss": lambda mse, mae: mse,
    "rmse_padded_loss": lambda mse, mae: torch.sqrt(mse),
    "rmse_mse_padded_loss": lambda mse, mae: torch.sqrt(mse) + mse,
    "l1_padded_loss": lambda mse, mae: mae,
    "combined_padded_loss": lambda mse, mae: torch.sqrt(mse) + mae,
}


def fock_loss(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt, loss_fn):
    name = getattr(loss_fn, "__name__", "")
    if _cuda(node_out) and name in DECOMPOSABLE:
        return _native.fock_loss(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt, name)
    nm = mask_table.index_select(0, node_pt)
    em = mask_table.index_select(0, edge_pt)
    return _ref.fock_loss(node_out, edge_out, node_t, edge_t, nm, em, loss_fn)


def fock_loss_stats_reference(node_out, edge_out, node_t, edge_t, mask_table, node_pt, edge_pt):
    """(sse_n, sae_n, cnt_n, sse_e, sae_e, cnt_e) - the sufficient statistics of the kernel."""
    nm = mask_table.index_select(0, node_pt).to(node_out.dtype)
    em = mask_table.index_select(0, edge_pt).to(edge_out.dtype)
    dn = (node_out - node_t) * nm
    de = (edge_out - edge_t) * em
    return torch.stack([(dn * dn).sum(), dn.abs().sum(), nm.sum(), (de * de).sum(), de.abs().sum(), em.sum()])
