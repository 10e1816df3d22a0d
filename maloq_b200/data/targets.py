"""Fock targets: Hamiltonian blocks -> coupled-basis labels per node and edge.

Mirrors the reference's ``Fock_Targets`` pipeline (``fock_utils/fock_targets_batched.py``):
matrix -> label rows (``matrix2label``) -> coupled basis (``get_net_out``) -> optional
per-element l=0 shift.  Synthetic Hamiltonians come from a frozen random-init teacher
model (:class:`Teacher`): its coupled outputs are mapped to blocks (``get_H`` +
``label2matrix``), symmetrised (H_ij <- (H_ij + H_ji^T) / 2), and then sent through the
forward pipeline, so targets are exactly equivariant and learnable.
"""

from __future__ import annotations

import numpy as np
import torch

from ..core.irreps import make_label_layout
from ..core.wigner3j import BasisTransform
from .batch import GraphSample, collate
from .labels import BlockSparseMatrix, PairTable, block_pointers, orbital_offsets


class FockLabeler:
    def __init__(self, orbital_basis, device="cpu", dtype=torch.float32):
        self.orbital_basis = {int(k): list(v) for k, v in orbital_basis.items()}
        self.layout = make_label_layout(self.orbital_basis)
        self.table = PairTable(self.layout)
        self.transform = BasisTransform(self.layout.out_js_list, dtype=dtype, device=device)
        self.device, self.dtype = torch.device(device), dtype
        self.pos_t, self.mask_t = self.table.torch_tables(self.device)

    @property
    def irreps(self):
        return self.layout.irreps_out

    @property
    def target_len(self):
        return self.layout.target_len

    def pairs(self, s: GraphSample):
        n = s.num_nodes
        rows = np.concatenate([s.src, np.arange(n)])
        cols = np.concatenate([s.dst, np.arange(n)])
        return rows, cols

    def _pt(self, s, rows, cols):
        return torch.as_tensor(self.table.pair_type(s.z[rows], s.z[cols]), device=self.device)

    def labels_from_blocks(self, s: GraphSample, bsm: BlockSparseMatrix):
        """Coupled labels (node_y [N, D], y [E, D]) of a block-sparse Hamiltonian whose
        blocks are ordered as ``pairs(s)``."""
        rows, cols = self.pairs(s)
        data = torch.as_tensor(bsm.data, device=self.device, dtype=self.dtype)
        ptr = torch.as_tensor(bsm.block_ptr, device=self.device)
        from ..ops import labels as lab_ops

        coupled = lab_ops.blocks_to_coupled(data, ptr, self._pt(s, rows, cols), self.pos_t, self.transform)
        E = s.num_edges
        return coupled[E:], coupled[:E]

    def blocks_from_labels(self, s: GraphSample, node_lab, edge_lab) -> BlockSparseMatrix:
        rows, cols = self.pairs(s)
        coupled = torch.cat([edge_lab, node_lab], 0).to(self.device, self.dtype)
        from ..ops import labels as lab_ops

        ptr_np = block_pointers(s.z, rows, cols, self.table)
        ptr = torch.as_tensor(ptr_np, device=self.device)
        data = lab_ops.coupled_to_blocks(coupled, ptr, self._pt(s, rows, cols), self.pos_t, self.transform,
                                         int(ptr_np[-1]))
        return BlockSparseMatrix(rows, cols, ptr_np, data.detach().cpu().numpy(), orbital_offsets(s.z, self.table))

    def symmetrize(self, s: GraphSample, bsm: BlockSparseMatrix) -> BlockSparseMatrix:
        """H_ij <- (H_ij + H_ji^T)/2 for every stored pair (the reverse pair must be stored)."""
        rows, cols = bsm.rows, bsm.cols
        n = s.num_nodes
        key = rows * n + cols
        rkey = cols * n + rows
        order = np.argsort(key)
        rev = order[np.searchsorted(key[order], rkey)]
        nz = self.table.norb[self.table.z_to_type[s.z]]
        out = bsm.data.copy()
        for b in range(len(rows)):
            a = bsm.data[bsm.block_ptr[b]:bsm.block_ptr[b + 1]].reshape(nz[rows[b]], nz[cols[b]])
            rb = rev[b]
            t = bsm.data[bsm.block_ptr[rb]:bsm.block_ptr[rb + 1]].reshape(nz[rows[rb]], nz[cols[rb]]).T
            out[bsm.block_ptr[b]:bsm.block_ptr[b + 1]] = (0.5 * (a + t)).ravel()
        return BlockSparseMatrix(rows, cols, bsm.block_ptr, out, bsm.orb_ptr)


class Teacher:
    """Frozen random-init backbone + Fock head producing coupled labels."""

    def __init__(self, model_kwargs, labeler: FockLabeler, seed=1234, device="cpu"):
        from ..models.backbone import eSEN_Backbone
        from ..models.heads import Fock_Irreps_Head

        g = torch.random.get_rng_state()
        torch.manual_seed(seed)
        kw = dict(model_kwargs)
        self.backbone = eSEN_Backbone(labeler.irreps, include_edges=True, **kw).to(device).eval()
        self.head = Fock_Irreps_Head(None, labeler.irreps, lmax=kw["lmax"], sphere_channels=kw["sphere_channels"],
                                     ls_list=labeler.layout.ls_list, reduce_node=False,
                                     open_shell=bool(kw.get("open_shell", False))).to(device).eval()
        torch.random.set_rng_state(g)
        for p in list(self.backbone.parameters()) + list(self.head.parameters()):
            p.requires_grad_(False)
        self.labeler, self.device = labeler, torch.device(device)

    @torch.no_grad()
    def hamiltonians(self, samples, chunk=16):
        """Symmetrised block-sparse Hamiltonians for ``samples`` (open shell: a list of the
        alpha and beta matrices per sample)."""
        out = []
        for i in range(0, len(samples), chunk):
            part = samples[i:i + chunk]
            b = collate(part, self.labeler.table).to(self.device)
            emb = self.backbone(b)
            n_all, e_all = self.head(emb, b)
            no, eo = 0, 0
            for s in part:
                per_spin = []
                for sp in range(n_all.shape[0]):
                    nl = n_all[sp, no:no + s.num_nodes]
                    el = e_all[sp, eo:eo + s.num_edges]
                    per_spin.append(self.labeler.symmetrize(s, self.labeler.blocks_from_labels(s, nl, el)))
                no += s.num_nodes
                eo += s.num_edges
                out.append(per_spin if len(per_spin) > 1 else per_spin[0])
        return out


def attach_scalar_targets(samples, teacher: Teacher, kind, seed=4321, chunk=16):
    """Energy or force targets of a frozen random-init energy/force head on the teacher's
    backbone (``kind``: "energies" or "forces"); sets ``sample.energy`` / ``sample.forces``.
    Energies are invariant and forces equivariant by construction, so they are learnable."""
    from ..models.heads import HELM_Energy_Head, HELM_Force_Head

    g = torch.random.get_rng_state()
    torch.manual_seed(seed)
    head = (HELM_Energy_Head if kind == "energies" else HELM_Force_Head)(teacher.backbone).to(teacher.device).eval()
    torch.random.set_rng_state(g)
    with torch.no_grad():
        for i in range(0, len(samples), chunk):
            part = samples[i:i + chunk]
            b = collate(part, teacher.labeler.table).to(teacher.device)
            out = head(teacher.backbone(b), b)
            if kind == "energies":
                for s, e in zip(part, out["energies"].double().cpu().numpy()):
                    s.energy = float(e)
            else:
                f = out["forces"].double().cpu().numpy()
                o = 0
                for s in part:
                    s.forces = f[o:o + s.num_nodes].copy()
                    o += s.num_nodes
    return samples


def attach_targets(samples, hamiltonians, labeler: FockLabeler, scale_shift=None):
    """Fill ``node_y``/``y`` ([spins, rows, D] float32, CPU) of every sample; a sample's
    Hamiltonian is one matrix, or a list of spin-channel matrices (open shell)."""
    for s, h in zip(samples, hamiltonians):
        nys, ys = [], []
        for hs in (h if isinstance(h, list) else [h]):
            ny, y = labeler.labels_from_blocks(s, hs)
            if scale_shift is not None:
                ny = scale_shift.shift(ny, s.z)
            nys.append(ny.cpu())
            ys.append(y.cpu())
        s.node_y = torch.stack(nys)
        s.y = torch.stack(ys)
    return samples


class ScaleShift:
    """Per-element mean of the l=0 node label entries, subtracted from targets (shift only,
    as the reference applies it: ``fock_targets_batched.py:1093-1194``)."""

    def __init__(self, labeler: FockLabeler, samples=None, means=None):
        irr = labeler.irreps
        idx, s = [], 0
        for it in irr:
            if it.l == 0:
                idx.append(s)
            s += it.dim
        self.scalar_idx = torch.tensor(idx, dtype=torch.long)
        self.means = means if means is not None else {}
        if samples is not None and means is None:
            acc, cnt = {}, {}
            for smp in samples:
                for z, row in zip(smp.z, smp.node_y[0]):
                    acc.setdefault(int(z), torch.zeros(len(idx)))
                    acc[int(z)] += row[self.scalar_idx].float()
                    cnt[int(z)] = cnt.get(int(z), 0) + 1
            self.means = {z: (acc[z] / cnt[z]) for z in acc}

    def _table(self, device, dtype):
        zmax = max(self.means) if self.means else 0
        t = torch.zeros(zmax + 1, len(self.scalar_idx), device=device, dtype=dtype)
        for z, v in self.means.items():
            t[z] = v.to(device, dtype)
        return t

    def shift(self, node_y, z):
        t = self._table(node_y.device, node_y.dtype)
        zt = torch.as_tensor(np.asarray(z), device=node_y.device)
        out = node_y.clone()
        out[:, self.scalar_idx.to(node_y.device)] -= t[zt]
        return out

    def unshift(self, node_y, z):
        t = self._table(node_y.device, node_y.dtype)
        zt = torch.as_tensor(np.asarray(z), device=node_y.device)
        out = node_y.clone()
        out[:, self.scalar_idx.to(node_y.device)] += t[zt]
        return out
