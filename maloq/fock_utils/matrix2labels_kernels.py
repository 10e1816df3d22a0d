"""Import-compatible module of the reference package (maloq.fock_utils.matrix2labels_kernels); the implementation lives in
:mod:`maloq_b200.data.labels and maloq_b200.ops.labels`. ``SparseBlockMatrix`` is :class:`BlockSparseMatrix`."""

from maloq_b200.data.labels import BlockSparseMatrix, PairTable, block_pointers  # noqa: F401
from maloq_b200.ops.labels import (  # noqa: F401
    blocks_to_coupled, coupled_to_blocks, labels_to_matrix, matrix_to_labels,
)

SparseBlockMatrix = BlockSparseMatrix
