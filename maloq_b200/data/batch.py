"""Graph samples and batches (replaces the reference's PyG ``Data``/``Batch`` objects).

A :class:`GraphSample` is one structure with its radius graph (dst-sorted edges) and,
optionally, its Fock targets in the coupled basis.  :func:`collate` concatenates samples
into a :class:`GraphBatch`; edges stay dst-sorted because molecules are contiguous.
Targets are stored per structure as ``[num_spins, rows, D]``; padding masks are not
materialised - they are ``mask_table[pair_type]`` (one bool row per element pair).
"""

from __future__ import annotations

import numpy as np
import torch

from .graph import dst_pointer, edge_attr_from_vec, radius_graph


class GraphSample:
    def __init__(self, z, pos, src, dst, edge_attr, charge=0, spin=1, node_y=None, y=None, cell=None):
        self.z = np.asarray(z, dtype=np.int64)
        self.pos = np.asarray(pos, dtype=np.float64)
        self.src, self.dst = np.asarray(src, dtype=np.int64), np.asarray(dst, dtype=np.int64)
        self.edge_attr = np.asarray(edge_attr, dtype=np.float64)
        self.charge, self.spin = int(charge), int(spin)
        self.node_y, self.y = node_y, y
        self.cell = cell
        self.energy = None  # total energy (scalar) for energy targets
        self.forces = None  # [N, 3] for force targets

    @property
    def num_nodes(self):
        return len(self.z)

    @property
    def num_edges(self):
        return len(self.src)


def make_sample(structure, cutoff) -> GraphSample:
    src, dst, vec = radius_graph(structure.pos, cutoff, structure.cell)
    return GraphSample(structure.z, structure.pos, src, dst, edge_attr_from_vec(vec), structure.charge,
                       structure.spin, cell=structure.cell)


_FIELDS_LONG = ("atomic_numbers", "atom_charge", "atom_spin", "batch", "edge_index", "dst_ptr", "src_z", "dst_z",
                "num_atoms_in_molecule", "node_pair_type", "edge_pair_type", "local_node_ids")


class GraphBatch:
    """Tensors of a batch of graphs.

    atomic_numbers/atom_charge/atom_spin/batch [N]; edge_index [2, E] (dst-sorted);
    edge_attr [E, 4] = [d, pos[src]-pos[dst]]; dst_ptr [N+1]; src_z/dst_z [E];
    node_y [S, N, D] and y [S, E, D] coupled-basis targets; node_pair_type [N] and
    edge_pair_type [E] index the layout's mask table.
    """

    def __init__(self, **kw):
        self.num_graphs = 1
        self.halo = None
        self.local_node_ids = None
        self.node_y = self.y = None
        for k, v in kw.items():
            setattr(self, k, v)

    @property
    def num_nodes(self):
        return int(self.atomic_numbers.shape[0])

    @property
    def num_edges(self):
        return int(self.edge_index.shape[1])

    def tensors(self):
        return {k: v for k, v in vars(self).items() if isinstance(v, torch.Tensor)}

    def to(self, device, non_blocking=False):
        out = GraphBatch(**{k: v for k, v in vars(self).items()})
        for k, v in self.tensors().items():
            setattr(out, k, v.to(device, non_blocking=non_blocking))
        return out

    def pin_memory(self):
        for k, v in self.tensors().items():
            setattr(self, k, v.pin_memory())
        return self

    def nbytes(self):
        return sum(v.numel() * v.element_size() for v in self.tensors().values())

    def __contains__(self, key):
        return getattr(self, key, None) is not None


def merge_samples(samples) -> GraphSample:
    """Disjoint union of molecule samples as one graph (a "supergraph"), for partitioning a
    batch of molecules over ranks: nodes and edges concatenated with offset indices, targets
    concatenated along the node / edge axis.  Per-atom charge, spin and molecule id are kept
    in ``atom_charge`` / ``atom_spin`` / ``atom_mol_id`` (reference: the batched targets of
    ``fock_utils/fock_targets_batched.py``, ``atom_mol_id``)."""
    off = 0
    src, dst, mol, ch, sp = [], [], [], [], []
    for g, s in enumerate(samples):
        src.append(s.src + off)
        dst.append(s.dst + off)
        mol.append(np.full(s.num_nodes, g, dtype=np.int64))
        ch.append(np.full(s.num_nodes, s.charge, dtype=np.int64))
        sp.append(np.full(s.num_nodes, s.spin, dtype=np.int64))
        off += s.num_nodes
    m = GraphSample(np.concatenate([s.z for s in samples]), np.concatenate([s.pos for s in samples]),
                    np.concatenate(src), np.concatenate(dst), np.concatenate([s.edge_attr for s in samples]),
                    samples[0].charge, samples[0].spin)
    m.atom_charge, m.atom_spin, m.atom_mol_id = np.concatenate(ch), np.concatenate(sp), np.concatenate(mol)
    if all(s.node_y is not None for s in samples):
        m.node_y = torch.cat([torch.as_tensor(s.node_y) for s in samples], dim=1)
        m.y = torch.cat([torch.as_tensor(s.y) for s in samples], dim=1)
    return m


def collate(samples, pair_table=None, target_dtype=torch.float32, float_dtype=torch.float32) -> GraphBatch:
    zs, pos, ch, sp, bt, srcs, dsts, eattr, nys, ys = [], [], [], [], [], [], [], [], [], []
    off = 0
    for g, s in enumerate(samples):
        zs.append(s.z)
        pos.append(s.pos)
        ch.append(np.full(s.num_nodes, s.charge))
        sp.append(np.full(s.num_nodes, s.spin))
        bt.append(np.full(s.num_nodes, g))
        srcs.append(s.src + off)
        dsts.append(s.dst + off)
        eattr.append(s.edge_attr)
        if s.node_y is not None:
            nys.append(s.node_y)
            ys.append(s.y)
        off += s.num_nodes
    z = np.concatenate(zs)
    src = np.concatenate(srcs)
    dst = np.concatenate(dsts)
    kw = dict(
        atomic_numbers=torch.as_tensor(z),
        pos=torch.as_tensor(np.concatenate(pos), dtype=float_dtype),
        atom_charge=torch.as_tensor(np.concatenate(ch)),
        atom_spin=torch.as_tensor(np.concatenate(sp)),
        batch=torch.as_tensor(np.concatenate(bt)),
        edge_index=torch.as_tensor(np.stack([src, dst])),
        edge_attr=torch.as_tensor(np.concatenate(eattr), dtype=float_dtype),
        dst_ptr=torch.as_tensor(dst_pointer(dst, len(z))),
        src_z=torch.as_tensor(z[src]),
        dst_z=torch.as_tensor(z[dst]),
        num_atoms_in_molecule=torch.as_tensor([s.num_nodes for s in samples]),
    )
    b = GraphBatch(**kw)
    b.num_graphs = len(samples)
    b.dst_ptr_host = kw["dst_ptr"].numpy()  # a host copy (not moved with the batch) for chunking
    if pair_table is not None:
        b.node_pair_type = torch.as_tensor(pair_table.pair_type(z, z))
        b.edge_pair_type = torch.as_tensor(pair_table.pair_type(z[src], z[dst]))
    if nys:
        b.node_y = torch.cat([torch.as_tensor(y) for y in nys], dim=1).to(target_dtype)
        b.y = torch.cat([torch.as_tensor(y) for y in ys], dim=1).to(target_dtype)
    if all(getattr(s, "energy", None) is not None for s in samples):
        b.energy = torch.as_tensor([float(s.energy) for s in samples], dtype=target_dtype)
    if all(getattr(s, "forces", None) is not None for s in samples):
        b.forces = torch.as_tensor(np.concatenate([np.asarray(s.forces) for s in samples]), dtype=target_dtype)
    return b


def batches_by_count(samples, batch_size, drop_last=True):
    out = []
    for i in range(0, len(samples), batch_size):
        chunk = samples[i:i + batch_size]
        if len(chunk) < batch_size and drop_last:
            break
        out.append(chunk)
    return out


def batches_by_atoms(samples, max_atoms):
    """Greedy first-fit-decreasing packing of samples into batches of <= max_atoms atoms
    (the atom-balanced batching of ``get_loader.py:732-1000``)."""
    order = sorted(range(len(samples)), key=lambda i: -samples[i].num_nodes)
    bins, loads = [], []
    for i in order:
        n = samples[i].num_nodes
        for k in range(len(bins)):
            if loads[k] + n <= max_atoms:
                bins[k].append(samples[i])
                loads[k] += n
                break
        else:
            bins.append([samples[i]])
            loads.append(n)
    return bins
