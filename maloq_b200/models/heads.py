"""Output heads: Hamiltonian-block (Fock) irreps head, energy head and force heads.

Reference: ``helm/esen_osh.py:521-1359``.  The Fock head keeps the reference's module
names (``lin_scalars_learnable``, ``node_lin_out_layers``, ``edge_lin_out_layers``,
``lin_out_layers``, ``parity_multiplier``) and the flat-weight layout of e3nn ``o3.Linear``
(one ``weight`` vector of ``mul_in * mul_out`` entries per degree, applied with a
``1/sqrt(mul_in)`` factor, a ``bias`` for scalar outputs only).  The per-spin work runs
through the grouped kernels in :mod:`maloq_b200.ops.head`.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch
import torch.nn as nn

from .. import ops
from ..core import irreps as ir
from .layers import GateActivation, SO2_Convolution, SO3_Linear
from .so3 import CoefficientMapping


@lru_cache(maxsize=None)
def second_moment_scale(name: str) -> float:
    """1 / sqrt(E[f(z)^2]) for z ~ N(0, 1) (Gauss-Hermite quadrature, 160 nodes).

    e3nn normalises gate activations to unit second moment; this is that constant for
    ``sigmoid`` and ``tanh`` computed by quadrature rather than sampling.
    """
    x, w = np.polynomial.hermite_e.hermegauss(160)
    f = {"sigmoid": lambda t: 1 / (1 + np.exp(-t)), "tanh": np.tanh}[name](x)
    m2 = float((w * f * f).sum() / w.sum())
    return 1.0 / math.sqrt(m2)


class E3Linear(nn.Module):
    """``mul_in x l -> mul_out x l`` linear map with e3nn's flat weight layout.

    Input/output layout [N, 2l+1, mul] (m outer, channel inner) - the transpose of e3nn's
    flattened layout, converted at the edges of the head.
    """

    def __init__(self, mul_in: int, mul_out: int, l: int, biases: bool = True):
        super().__init__()
        self.mul_in, self.mul_out, self.l = mul_in, mul_out, l
        self.weight = nn.Parameter(torch.randn(mul_in * mul_out))
        nb = mul_out if (biases and l == 0) else 0
        self.bias = nn.Parameter(torch.zeros(nb))
        self.register_buffer("output_mask", torch.ones(mul_out * (2 * l + 1)) if mul_in > 0 else torch.zeros(mul_out * (2 * l + 1)))

    def weight_matrix(self):
        """[mul_out, mul_in] already scaled by 1/sqrt(mul_in) (a torch ``Linear`` weight)."""
        return self.weight.view(self.mul_in, self.mul_out).t() / math.sqrt(self.mul_in)

    def forward(self, x):
        if self.mul_out == 0:
            return x.new_zeros(x.shape[0], 2 * self.l + 1, 0)
        return ops.linear(x, self.weight_matrix(), self.bias if self.bias.numel() else None)


class IrrepsGate(nn.Module):
    """Parameter-free gate: gated irreps times act(gate scalar), act normalised to unit
    second moment (the e3nn ``Gate`` with empty scalar part)."""

    def __init__(self, act: str):
        super().__init__()
        self.act = act
        self.scale = second_moment_scale(act)


class Fock_Irreps_Head(nn.Module):
    """Maps backbone irreps to per-node and per-edge Hamiltonian-block labels (coupled basis)."""

    def __init__(self, irreps_in=None, irreps_out=None, lmax=4, sphere_channels=128, reduce_edge=False, ls_list=None,
                 open_shell=False, reduce_node=False, reduce_node_intra=False, orbital_basis=None):
        super().__init__()
        self.sphere_channels, self.lmax = sphere_channels, lmax
        self.reduce_node, self.reduce_node_intra, self.reduce_edge = reduce_node, reduce_node_intra, reduce_edge
        self.irreps_out = ir.Irreps(irreps_out)
        self.ls_list = [int(l) for l in ls_list]
        self.num_spins = 2 if open_shell else 1
        C = sphere_channels
        not_antisym = not reduce_edge
        perms = {}
        if reduce_node:
            self.irreps_nodereduced = ir.reduced_node_irreps(self.ls_list, reduce_node_intra)
            red2all = ir.reduced_to_all_indices(self.ls_list, reduce_node_intra)
            self.register_buffer("parity_multiplier",
                                 torch.tensor(ir.parity_multiplier(self.ls_list, reduce_node_intra), dtype=torch.float32))
            perms["node"] = ir.sorted_to_original_permutation(self.irreps_nodereduced)
        if reduce_edge:
            if not reduce_node:
                raise NotImplementedError("reduce_edge without reduce_node is not supported (as in the reference)")
            a, b, flips, offa, offb = ir.edge_reduced_irreps(self.ls_list)
            self.irreps_edgereduced_alpha, self.irreps_edgereduced_beta = a, b
            self.parity_flip_indices, self.off_diag_alpha, self.off_diag_beta = flips, offa, offb
            perms["edge_alpha"] = ir.sorted_to_original_permutation(a)
            perms["edge_beta"] = ir.sorted_to_original_permutation(b)
            self.remix = ir.subspace_remix_permutation(a, b, self.ls_list)
        elif reduce_node:
            perms["edge"] = ir.sorted_to_original_permutation(self.irreps_out)
        else:
            perms["common"] = ir.sorted_to_original_permutation(self.irreps_out)
        self.output_permutation = perms

        n_gated = C * lmax
        self.lin_scalars_learnable = nn.ModuleList()
        self.gate = nn.ModuleList()
        if reduce_node and reduce_edge:
            self.node_lin_out_layers = nn.ModuleList()
            self.edge_lin_out_layers = nn.ModuleDict({"alpha": nn.ModuleList(), "beta": nn.ModuleList()})
        elif reduce_node:
            self.node_lin_out_layers = nn.ModuleList()
            self.edge_lin_out_layers = nn.ModuleList()
        else:
            self.lin_out_layers = nn.ModuleList()

        def per_l(irreps, biases):
            return nn.ModuleList([E3Linear(C, irreps.count(l), l, biases) for l in range(lmax + 1)])

        for _ in range(self.num_spins):
            self.lin_scalars_learnable.append(E3Linear(C, C + n_gated, 0, biases=not_antisym))
            self.gate.append(IrrepsGate("sigmoid" if not_antisym else "tanh"))
            if reduce_node and reduce_edge:
                self.node_lin_out_layers.append(per_l(self.irreps_nodereduced, True))
                self.edge_lin_out_layers["alpha"].append(per_l(self.irreps_edgereduced_alpha, not_antisym))
                self.edge_lin_out_layers["beta"].append(per_l(self.irreps_edgereduced_beta, not_antisym))
            elif reduce_node:
                self.node_lin_out_layers.append(per_l(self.irreps_nodereduced, True))
                self.edge_lin_out_layers.append(per_l(self.irreps_out, True))
            else:
                self.lin_out_layers.append(per_l(self.irreps_out, True))

        # one gather per output kind: label[k] = mult[k] * sorted_out[idx[k]] (idx -1 -> 0)
        if reduce_node:
            pn = np.asarray(perms["node"])
            r2a = np.asarray(red2all)
            idx = np.where(r2a >= 0, pn[np.clip(r2a, 0, None)], -1)
            self.register_buffer("_node_gather", torch.tensor(idx, dtype=torch.long), persistent=False)
        else:
            self.register_buffer("_node_gather", torch.tensor(perms["common"], dtype=torch.long), persistent=False)
        if not reduce_edge:
            key = "edge" if reduce_node else "common"
            self.register_buffer("_edge_gather", torch.tensor(perms[key], dtype=torch.long), persistent=False)

    # ------------------------------------------------------------------
    def _layers(self, kind, spin):
        if not self.reduce_node:
            return self.lin_out_layers[spin]
        if kind == "node":
            return self.node_lin_out_layers[spin]
        if kind == "edge":
            return self.edge_lin_out_layers[spin]
        return self.edge_lin_out_layers["alpha" if kind == "edge_alpha" else "beta"][spin]

    def process(self, x, kind, spin):
        """[N, (L+1)^2, C] -> outputs grouped by l (sorted irreps order), [N, D_sorted]."""
        lin_s = self.lin_scalars_learnable[spin]
        layers = self._layers(kind, spin)
        return ops.fock_head_process(x, lin_s.weight_matrix(), lin_s.bias if lin_s.bias.numel() else None,
                                     [(lay.weight_matrix() if lay.mul_out else None,
                                       lay.bias if lay.bias.numel() else None) for lay in layers],
                                     self.gate[spin].act, self.gate[spin].scale, self.reduce_edge and kind != "node")

    def node_labels(self, node_emb, spin=0):
        """Node label rows of one spin channel (the node part of ``forward``)."""
        n_sorted = self.process(node_emb, "node", spin)
        return ops.gather_scale(n_sorted, self._node_gather, self.parity_multiplier if self.reduce_node else None)

    def edge_labels(self, edge_emb, spin=0):
        """Edge label rows of one spin channel for any subset of edge rows (row-wise; the
        ``reduce_edge`` head pairs edges and is not row-wise)."""
        if self.reduce_edge:
            raise ValueError("edge_labels is row-wise; the reduce_edge head needs all edges")
        return ops.gather_scale(self.process(edge_emb, "edge", spin), self._edge_gather, None)

    def forward(self, emb, batch=None):
        node_emb, edge_emb = emb["node_embeddings"], emb["edge_embeddings"]
        edge_index = emb["edge_index"]
        node_outs, edge_outs = [], []
        if self.reduce_edge:
            alpha, beta, half_mask, rev = self.half_antisym_edge_pairs(edge_emb.to(node_emb.dtype), edge_index,
                                                                       node_emb.shape[0])
        for spin in range(self.num_spins):
            n_sorted = self.process(node_emb, "node", spin)
            if self.reduce_node:
                node_out = ops.gather_scale(n_sorted, self._node_gather, self.parity_multiplier)
            else:
                node_out = ops.gather_scale(n_sorted, self._node_gather, None)
            if self.reduce_edge:
                oa = self.process(alpha, "edge_alpha", spin)
                ob = self.process(beta, "edge_beta", spin)
                oa, ob = self.half_edges_to_full(rev, half_mask, oa, ob)
                pa, pb, ia, ib, remix, sign = self._reduce_edge_tables(oa.device, oa.dtype, oa.shape[1] + ob.shape[1])
                oa, ob = oa.index_select(1, pa), ob.index_select(1, pb)
                va, vb = oa.index_select(1, ia), ob.index_select(1, ib)
                oa = oa.index_copy(1, ia, va + vb)
                ob = ob.index_copy(1, ib, va - vb)
                edge_out = torch.cat([oa, ob], dim=-1).index_select(1, remix) * sign
            elif emb.get("edge_chunks"):
                # row-wise over edges: one chunk at a time (recomputed in backward)
                def rows(x, spin=spin):
                    return ops.gather_scale(self.process(x.to(node_emb.dtype), "edge", spin), self._edge_gather, None)

                if torch.is_grad_enabled():
                    from torch.utils.checkpoint import checkpoint

                    parts = [checkpoint(rows, edge_emb[e0:e1], use_reentrant=False) for e0, e1 in emb["edge_chunks"]]
                else:
                    parts = [rows(edge_emb[e0:e1]) for e0, e1 in emb["edge_chunks"]]
                edge_out = torch.cat(parts, 0)
            else:
                edge_out = ops.gather_scale(self.process(edge_emb, "edge", spin), self._edge_gather, None)
            node_outs.append(node_out)
            edge_outs.append(edge_out)
        return torch.stack(node_outs, 0), torch.stack(edge_outs, 0)

    def _reduce_edge_tables(self, device, dtype, width):
        """Index tables of the reduce_edge remix on ``device``, built once (a per-call copy from
        host lists would wait for the device)."""
        key = (str(device), dtype, width)
        cache = self.__dict__.setdefault("_tables", {})
        if key not in cache:
            flips = torch.as_tensor(self.parity_flip_indices, dtype=torch.long)
            sign = torch.ones(width, dtype=dtype).index_fill(0, flips, -1.0)
            lt = lambda v: torch.as_tensor(v, dtype=torch.long).to(device)
            cache[key] = (lt(self.output_permutation["edge_alpha"]), lt(self.output_permutation["edge_beta"]),
                          lt(self.off_diag_alpha), lt(self.off_diag_beta), lt(self.remix), sign.to(device))
        return cache[key]

    @staticmethod
    def reverse_edge_indices(edge_index, num_nodes=None):
        """rev[e] = the edge with the endpoints of e swapped (every edge has one).  ``num_nodes``
        (known on the host) avoids reading the largest index back from the device."""
        if num_nodes is None:
            num_nodes = int(edge_index.max()) + 1 if edge_index.numel() else 1
        n = int(num_nodes)
        _, po = torch.sort(edge_index[0] * n + edge_index[1])
        _, pf = torch.sort(edge_index[1] * n + edge_index[0])
        return pf[torch.argsort(po)]

    def half_antisym_edge_pairs(self, edge_emb, edge_index, num_nodes=None):
        """Symmetric/antisymmetric combinations for the canonical half of the edge pairs (the
        edges e with e < rev[e]: exactly half of them, so they are selected by a stable sort
        rather than a boolean mask - no host synchronisation).  Returns (a + b, a - b, the
        half's edge ids, rev)."""
        rev = self.reverse_edge_indices(edge_index, num_nodes)
        E = edge_index.shape[1]
        first = torch.arange(E, device=edge_index.device) < rev
        half = torch.argsort((~first).to(torch.int8), stable=True)[: E // 2]
        a, b = edge_emb.index_select(0, half), edge_emb.index_select(0, rev.index_select(0, half))
        return a + b, a - b, half, rev

    @staticmethod
    def half_edges_to_full(rev, half, oa, ob):
        """Full edge rows from the half's outputs: the half's rows and, at their reverse edges,
        the same alpha rows and negated beta rows (``half``: edge ids)."""
        E = rev.shape[0]
        flipped = rev.index_select(0, half)
        fa = oa.new_zeros((E,) + oa.shape[1:]).index_copy(0, half, oa).index_copy(0, flipped, oa)
        fb = ob.new_zeros((E,) + ob.shape[1:]).index_copy(0, half, ob).index_copy(0, flipped, -ob)
        return fa, fb


class _ConvHeadBase(nn.Module):
    """One extra Edgewise-style convolution on node embeddings, summed into nodes."""

    def __init__(self, backbone, out_channels):
        super().__init__()
        self.sphere_channels, self.hidden_channels = backbone.sphere_channels, backbone.hidden_channels
        self.lmax, self.mmax = backbone.lmax, backbone.mmax
        self.mappingReduced = CoefficientMapping(self.lmax, self.mmax)
        self.act = GateActivation(self.lmax, self.mmax, self.hidden_channels, outer_dim="m", mapping=self.mappingReduced)
        self.concat_size = 2
        self.so2_conv_1 = SO2_Convolution(2 * self.sphere_channels, self.hidden_channels, self.lmax, self.mmax,
                                          self.mappingReduced, internal_weights=False,
                                          edge_channels_list=backbone.edge_channels_list,
                                          extra_m0_output_channels=self.lmax * self.hidden_channels)
        self.so2_conv_2 = SO2_Convolution(self.hidden_channels, out_channels, self.lmax, self.mmax,
                                          self.mappingReduced, internal_weights=True)

    @property
    def mapping(self):
        """The coefficient mapping under the name the Edgewise ops read (``mappingReduced`` is
        the reference's attribute name)."""
        return self.mappingReduced

    def conv(self, emb):
        xe = emb["x_edge"]
        if hasattr(xe, "full"):  # chunked backbones hand over the lazy edge features
            xe = xe.full()
        graph = emb["graph"]
        if graph.chunks is not None:  # one pass over all edges (the head is small)
            graph = graph.whole()
        return ops.edgewise(self, emb["node_embeddings"], None, xe, graph, "node")


class HELM_Energy_Head(_ConvHeadBase):
    """Per-molecule energy: conv -> l=0 -> MLP -> sum over atoms (``esen_osh.py:1139-1254``)."""

    def __init__(self, backbone):
        super().__init__(backbone, backbone.sphere_channels)
        h = 2 * self.sphere_channels
        self.linear = nn.Sequential(nn.Linear(self.sphere_channels, h, bias=True), nn.SiLU(), nn.Linear(h, 1, bias=True))

    def forward(self, emb, batch):
        x = self.conv(emb)
        e_atom = self.linear(x[:, 0]).squeeze(-1)
        n_mol = batch.num_graphs
        return {"energies": e_atom.new_zeros(n_mol).index_add_(0, batch.batch, e_atom)}


class HELM_Force_Head(_ConvHeadBase):
    """Forces from the l=1 output of one extra convolution (``esen_osh.py:1258-1342``)."""

    def __init__(self, backbone):
        super().__init__(backbone, 1)

    def forward(self, emb, batch):
        x = self.conv(emb)
        return {"forces": x[:, 1:4, 0]}


class HELM_Simple_Force_Head(nn.Module):
    """SO3 linear on l <= 1 -> l = 1 components (``esen_osh.py:1346-1359``)."""

    def __init__(self, backbone):
        super().__init__()
        self.linear = SO3_Linear(backbone.sphere_channels, 1, lmax=1)

    def forward(self, emb, batch):
        f = self.linear(emb["node_embeddings"][:, :4])
        return {"forces": f[:, 1:4].reshape(-1, 3).contiguous()}
