"""Hamiltonian blocks <-> label rows (uncoupled basis), block-sparse matrices.

A Hamiltonian of a structure is kept as a :class:`BlockSparseMatrix`: one dense
``n_orb(i) x n_orb(j)`` block per stored atom pair (i, j), back to back in ``data``.
(Reference: the dense and block-sparse CuPy kernels ``fock_utils/matrix2labels_kernels.py``
and the ``SparseBlockMatrix`` tuple there.)  A label row of pair (i, j) has ``target_len``
entries; entry ``out0 + r * (c1 - c0) + c`` of a template item ``(r0, r1, c0, c1, out0)``
holds ``block[r0 + r, c0 + c]``; entries outside the template are padding (0).

:class:`PairTable` turns the layout's template into one gather table per element pair
(``pos[type, k]`` = flat position inside the block, -1 for padding) so that the
conversion is a single gather (``matrix_to_labels``) or scatter (``labels_to_matrix``);
the CUDA kernels in ``ops/csrc/labels.cu`` use the same table.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..core.irreps import LabelLayout


class PairTable:
    """Per element-pair gather positions and masks for a label layout."""

    def __init__(self, layout: LabelLayout, max_z: int = 100):
        self.layout = layout
        self.elements = sorted(layout.orbitals_per_element)
        self.z_to_type = np.full(max_z + 1, -1, dtype=np.int64)
        for t, z in enumerate(self.elements):
            self.z_to_type[z] = t
        nt = len(self.elements)
        D = layout.target_len
        pos = np.full((nt * nt, D), -1, dtype=np.int64)
        for a, zi in enumerate(self.elements):
            for b, zj in enumerate(self.elements):
                ncol = layout.orbitals_per_element[zj]
                for r0, r1, c0, c1, o in layout.template[(zi, zj)]:
                    nc = c1 - c0
                    for r in range(r1 - r0):
                        for c in range(nc):
                            pos[a * nt + b, o + r * nc + c] = (r0 + r) * ncol + (c0 + c)
        self.pos = pos
        self.mask = pos >= 0
        self.n_types = nt
        self.norb = np.array([layout.orbitals_per_element[z] for z in self.elements], dtype=np.int64)

    def pair_type(self, zi, zj):
        return self.z_to_type[np.asarray(zi)] * self.n_types + self.z_to_type[np.asarray(zj)]

    def torch_tables(self, device):
        return (torch.as_tensor(self.pos, device=device), torch.as_tensor(self.mask, device=device))


@dataclass
class BlockSparseMatrix:
    """Block-sparse Hamiltonian: ``rows``/``cols`` atom ids of each block, ``block_ptr``
    data offsets (len nb+1), ``data`` flat values, ``orb_ptr`` per-atom orbital offsets."""

    rows: np.ndarray
    cols: np.ndarray
    block_ptr: np.ndarray
    data: np.ndarray
    orb_ptr: np.ndarray

    @property
    def n_orb(self):
        return int(self.orb_ptr[-1])

    def to_dense(self):
        n = self.n_orb
        M = np.zeros((n, n), dtype=self.data.dtype)
        for b in range(len(self.rows)):
            i, j = self.rows[b], self.cols[b]
            r0, r1, c0, c1 = self.orb_ptr[i], self.orb_ptr[i + 1], self.orb_ptr[j], self.orb_ptr[j + 1]
            M[r0:r1, c0:c1] = self.data[self.block_ptr[b]:self.block_ptr[b + 1]].reshape(r1 - r0, c1 - c0)
        return M

    def to_scipy_csr(self):
        import scipy.sparse as sp

        rr, cc, vv = [], [], []
        for b in range(len(self.rows)):
            i, j = self.rows[b], self.cols[b]
            r0, r1, c0, c1 = self.orb_ptr[i], self.orb_ptr[i + 1], self.orb_ptr[j], self.orb_ptr[j + 1]
            g = np.meshgrid(np.arange(r0, r1), np.arange(c0, c1), indexing="ij")
            rr.append(g[0].ravel())
            cc.append(g[1].ravel())
            vv.append(self.data[self.block_ptr[b]:self.block_ptr[b + 1]])
        n = self.n_orb
        return sp.coo_matrix((np.concatenate(vv), (np.concatenate(rr), np.concatenate(cc))), shape=(n, n)).tocsr()

    def save_npz(self, path):
        """The matrix as a scipy CSR ``.npz`` (``scipy.sparse.load_npz`` reads it back; the
        reference's inference output format)."""
        import scipy.sparse as sp

        sp.save_npz(path, self.to_scipy_csr())
        return path

    @staticmethod
    def from_dense(M, rows, cols, orb_ptr):
        sizes = (orb_ptr[rows + 1] - orb_ptr[rows]) * (orb_ptr[cols + 1] - orb_ptr[cols])
        ptr = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        data = np.empty(int(ptr[-1]), dtype=M.dtype)
        for b, (i, j) in enumerate(zip(rows, cols)):
            data[ptr[b]:ptr[b + 1]] = M[orb_ptr[i]:orb_ptr[i + 1], orb_ptr[j]:orb_ptr[j + 1]].ravel()
        return BlockSparseMatrix(np.asarray(rows), np.asarray(cols), ptr, data, np.asarray(orb_ptr))


def orbital_offsets(z, table: PairTable):
    n = table.norb[table.z_to_type[np.asarray(z)]]
    return np.concatenate([[0], np.cumsum(n)]).astype(np.int64)


def block_pointers(z, rows, cols, table: PairTable):
    nz = table.norb[table.z_to_type[np.asarray(z)]]
    sizes = nz[rows] * nz[cols]
    return np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)


def matrix_to_labels(data, block_ptr, pair_type, pos_table):
    """labels[b, k] = data[block_ptr[b] + pos[pair_type[b], k]] (0 where pos < 0). Torch, any device."""
    from ..ops import labels as lab

    return lab.matrix_to_labels(data, block_ptr, pair_type, pos_table)


def labels_to_matrix(labels, block_ptr, pair_type, pos_table, n_data):
    from ..ops import labels as lab

    return lab.labels_to_matrix(labels, block_ptr, pair_type, pos_table, n_data)
