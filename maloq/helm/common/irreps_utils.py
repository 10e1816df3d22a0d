"""Import-compatible module of the reference package (maloq.helm.common.irreps_utils); the implementation lives in
:mod:`maloq_b200.core.irreps`."""

from maloq_b200.core.irreps import (  # noqa: F401
    Irreps, edge_reduced_irreps, parity_multiplier, product_irreps, product_ls, reduced_node_irreps,
    reduced_to_all_indices, subspace_remix_permutation,
)
