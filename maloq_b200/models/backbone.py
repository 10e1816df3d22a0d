"""SO(2)-equivariant eSEN backbone (HELM) with m-truncated edge-frame rotations.

Reference: ``helm/esen_osh.py:57-517`` (backbone), ``helm/esen_block.py`` (blocks),
``helm/nn/embedding.py`` (edge-degree embedding).  Differences by design:

* the per-edge rotation is built once per forward as a compact m-truncated
  matrix ``rot`` [E, R, (L+1)^2] (R = m-major rows with |m| <= mmax), which also performs
  the l->m reordering; the reverse rotation is its transpose.  This makes ``mmax < lmax``
  work (the reference needs ``mmax == lmax``);
* the roll angle gamma is 0 instead of random: the SO(2) layers commute with rolls about
  the edge axis, so the output does not depend on it;
* in graph-partitioned mode the source-node features of an edge may live on another
  GPU; the edge kernels read them through a :class:`maloq_b200.parallel.halo.HaloPlan`.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..core import sph
from .layers import (
    EnvelopedBesselBasis,
    GateActivation,
    GaussianSmearing,
    RadialMLP,
    SO2_Convolution,
    SO3_Linear,
    get_normalization_layer,
)
from .so3 import CoefficientMapping


class Edgewise(nn.Module):
    """Message passing: gather, rotate into the edge frame, SO(2) conv, gate, SO(2) conv,
    rotate back, then sum over incoming edges (node path) or keep per edge (edge path).

    Reference ``helm/esen_block.py:34-258``.
    """

    def __init__(self, sphere_channels, hidden_channels, lmax, mmax, edge_channels_list, mapping,
                 message_type="source-target"):
        super().__init__()
        self.sphere_channels, self.hidden_channels = sphere_channels, hidden_channels
        self.lmax, self.mmax = lmax, mmax
        self.mapping = mapping
        self.act = GateActivation(lmax, mmax, hidden_channels, outer_dim="m", mapping=mapping)
        if message_type == "source-target-message":
            self.concat_size = 3
        elif message_type == "source-target":
            self.concat_size = 2
        else:
            raise ValueError(f"unknown message_type {message_type!r}")
        self.so2_conv_1 = SO2_Convolution(self.concat_size * sphere_channels, hidden_channels, lmax, mmax, mapping,
                                          internal_weights=False, edge_channels_list=edge_channels_list,
                                          extra_m0_output_channels=lmax * hidden_channels)
        self.so2_conv_2 = SO2_Convolution(hidden_channels, sphere_channels, lmax, mmax, mapping,
                                          internal_weights=True)

    def forward(self, x_node, x_message_edge, x_edge, graph, node_or_edge):
        return ops.edgewise(self, x_node, x_message_edge if self.concat_size == 3 else None, x_edge, graph,
                            node_or_edge)


class SpectralAtomwise(nn.Module):
    """Gate scalars from l=0, SO3_Linear, gate, SO3_Linear (``esen_block.py:261-298``)."""

    def __init__(self, sphere_channels, hidden_channels, lmax, mmax):
        super().__init__()
        self.lmax = lmax
        self.hidden_channels = hidden_channels
        self.scalar_mlp = nn.Sequential(nn.Linear(sphere_channels, lmax * hidden_channels, bias=True), nn.SiLU())
        self.so3_linear_1 = SO3_Linear(sphere_channels, hidden_channels, lmax)
        self.act = GateActivation(lmax, lmax, hidden_channels, outer_dim="l")
        self.so3_linear_2 = SO3_Linear(hidden_channels, sphere_channels, lmax)

    def forward(self, x, residual=None):
        """``residual`` is added to the output (in the second SO3 linear's GEMM epilogue on the
        kernel path).  The hidden activations between the two SO3 linears are bf16 on the kernel
        path (they only feed the next GEMM)."""
        lin = self.scalar_mlp[0]
        s1 = self.so3_linear_1
        h, pre = ops.so3_linear_scalar(x, s1.weight, s1.bias, self.lmax, torch.bfloat16, lin.weight, lin.bias)
        h = ops.gate_silu(pre, h, self.act.expand_index, self.lmax)  # = self.act(silu(pre), h)
        return self.so3_linear_2(h, residual=residual)


class eSEN_Block(nn.Module):
    """Node path: norm -> Edgewise -> +res -> norm -> atomwise -> +res.
    Edge path: Edgewise -> norm -> +res -> norm -> atomwise -> +res (``esen_block.py:301-419``)."""

    def __init__(self, sphere_channels, hidden_channels, lmax, mmax, mapping, edge_channels_list,
                 norm_type="rms_norm_sh", message_type="source-target", node_or_edge="node"):
        super().__init__()
        self.node_or_edge = node_or_edge
        self.norm_1 = get_normalization_layer(norm_type, lmax, sphere_channels)
        self.norm_2 = get_normalization_layer(norm_type, lmax, sphere_channels)
        self.edge_wise = Edgewise(sphere_channels, hidden_channels, lmax, mmax, edge_channels_list, mapping, message_type)
        self.atom_wise = SpectralAtomwise(sphere_channels, hidden_channels, lmax, mmax)

    def forward(self, x_node, x_edge_emb, x_edge, graph):
        if graph.chunks is not None:
            return self._forward_chunked(x_node, x_edge_emb, x_edge, graph)
        if self.node_or_edge == "node":
            h = self.norm_1(x_node)
            h = self.edge_wise(h, x_edge_emb, x_edge, graph, "node")
            h, res = self.norm_2(h, residual=x_node, out_dtype=torch.bfloat16)  # res = h + x_node
            return self.atom_wise(h, residual=res)
        h = self.edge_wise(x_node, x_edge_emb, x_edge, graph, "edge")
        h = self.norm_1(h)
        h, res = self.norm_2(h, residual=x_edge_emb, out_dtype=torch.bfloat16)
        return self.atom_wise(h, residual=res)

    # ------------------------------------------------------------------ edge-chunked execution
    def _forward_chunked(self, x_node, x_edge_emb, x_edge, graph):
        """The same block over dst-contiguous edge chunks.  With gradients each chunk is
        recomputed in backward (only its inputs, views of the layer inputs, are kept), so the
        per-edge working set is bounded by the chunk size; without gradients the edge block
        overwrites the edge stream chunk by chunk.  Halo rows are exchanged once per block
        (``HaloPlan.materialize``) and shared by the chunks.  ``x_edge`` may be an
        :class:`EdgeInputs` (rows computed per chunk).  The edge stream keeps the dtype it
        arrives in (bf16 storage by default; every chunk computes in the node stream's dtype)."""
        grad = torch.is_grad_enabled()
        run = _checkpointed if grad else (lambda f, *a: f(*a))
        if self.node_or_edge == "node":
            h = self.norm_1(x_node)
            hx = graph.halo.materialize(h) if graph.halo is not None else h
            outs = [run(self._node_rows, hx, _rows(x_edge_emb, e0, e1), x_edge, e0, e1, graph.chunk_graph(i))
                    for i, (e0, e1, _, _) in enumerate(graph.chunks)]
            h, res = self.norm_2(torch.cat(outs, 0), residual=x_node, out_dtype=torch.bfloat16)
            return self.atom_wise(h, residual=res)
        xn = graph.halo.materialize(x_node) if graph.halo is not None else x_node
        if not grad:
            for i, (e0, e1, _, _) in enumerate(graph.chunks):
                x_edge_emb[e0:e1] = self._edge_rows(xn, x_edge_emb[e0:e1], x_edge, e0, e1, graph.chunk_graph(i))
            return x_edge_emb
        outs = [run(self._edge_rows, xn, x_edge_emb[e0:e1], x_edge, e0, e1, graph.chunk_graph(i))
                for i, (e0, e1, _, _) in enumerate(graph.chunks)]
        return torch.cat(outs, 0)

    def _node_rows(self, hx, xm, x_edge, e0, e1, sub):
        return self.edge_wise(hx, None if xm is None else xm.to(hx.dtype), x_edge[e0:e1], sub, "node")

    def _edge_rows(self, xn, xee, x_edge, e0, e1, sub):
        x_in = xee.to(xn.dtype)  # compute dtype of the node stream
        h = self.edge_wise(xn, x_in, x_edge[e0:e1], sub, "edge")
        h = self.norm_1(h)
        h, res = self.norm_2(h, residual=x_in, out_dtype=torch.bfloat16)
        return self.atom_wise(h, residual=res).to(xee.dtype)


class EdgeInputs:
    """Edge features ``[src embedding | Gaussian(d) | dst embedding]`` computed for a row range
    on use (``x_edge[e0:e1]``), so chunked execution never holds them for every edge."""

    def __init__(self, backbone, batch, dist):
        self.bb, self.batch, self.dist = backbone, batch, dist

    def __getitem__(self, sl):
        e0, e1 = sl.start or 0, sl.stop
        b, bb = self.batch, self.bb
        return torch.cat([ops.embedding(b.src_z[e0:e1], bb.source_embedding.weight),
                          bb.distance_expansion(self.dist[e0:e1]),
                          ops.embedding(b.dst_z[e0:e1], bb.target_embedding.weight)], dim=1)

    def full(self):
        return self[0:self.dist.shape[0]]


def _rows(x, e0, e1):
    return None if x is None else x[e0:e1]


def _checkpointed(fn, *args):
    from torch.utils.checkpoint import checkpoint

    return checkpoint(fn, *args, use_reentrant=False)


class EdgeDegreeEmbedding(nn.Module):
    """Radial MLP -> m = 0 coefficients -> rotate back -> sum/rescale into nodes, or per edge.

    Reference ``helm/nn/embedding.py:17-141``.
    """

    def __init__(self, sphere_channels, lmax, mmax, edge_channels_list, rescale_factor, mapping):
        super().__init__()
        self.sphere_channels, self.lmax = sphere_channels, lmax
        self.m0 = mapping.m_size[0]
        self.rad_func = RadialMLP(list(edge_channels_list) + [self.m0 * sphere_channels])
        self.rescale_factor = rescale_factor

    def forward(self, x_node, x_edge, graph, node_or_edge="node"):
        e = self.rad_func(x_edge).view(-1, self.m0, self.sphere_channels)
        if node_or_edge == "node":
            return ops.rotate_back_m0_scatter(e, graph, x_node, 1.0 / self.rescale_factor)
        return ops.rotate_back_m0(e, graph)


def _model_frame(edge_attr):
    """Edge vectors in the model frame: columns [d, x, y, z] -> (y, z, x), polar axis = input z
    (slices, so no index tensor is copied to the device per call)."""
    return torch.cat([edge_attr[:, 2:4], edge_attr[:, 1:2]], dim=1)


class Graph:
    """Per-forward graph data shared by all layers.

    ``src``/``dst``: edge endpoints (local node ids; with a partition, ``src`` may index the
    halo); ``rot``: m-truncated rotation; ``dst_ptr``: CSR offsets of edges sorted by
    ``dst`` (edges must be dst-sorted); ``num_nodes``; ``halo``: optional HaloPlan.
    """

    def __init__(self, src, dst, rot, dst_ptr, num_nodes, lmax, mmax, halo=None):
        self.src, self.dst, self.rot, self.dst_ptr = src, dst, rot, dst_ptr
        self.num_nodes, self.lmax, self.mmax, self.halo = num_nodes, lmax, mmax, halo
        self.cache = {}
        # node-path output rows: the scatter writes rows [0, num_out) through out_ptr / dst_out
        # (all nodes here; one chunk's destination range in a sub-graph)
        self.out_ptr, self.dst_out, self.num_out = dst_ptr, dst, num_nodes
        self.chunks = None  # [(e0, e1, n0, n1)] for edge-chunked execution
        self.rot_fn = None  # (e0, e1) -> rotations of those edges, when rot is not stored

    def whole(self):
        """The unchunked graph (rotations computed if they are not stored)."""
        if self.chunks is None:
            return self
        g = Graph(self.src, self.dst, self.rot if self.rot is not None else self.rot_fn(0, self.src.shape[0]),
                  self.dst_ptr, self.num_nodes, self.lmax, self.mmax, self.halo)
        g.num_nodes_ext = getattr(self, "num_nodes_ext", None) or self.num_nodes
        return g

    def chunk_graph(self, i):
        """Sub-graph of chunk ``i``.  With gradients the sub-graphs are built once per forward
        and shared by every layer (their cached source CSRs are reused in backward); without
        gradients they are built on use, and with ``rot_fn`` set the chunk's rotations are
        computed then instead of being held for every edge."""
        if torch.is_grad_enabled() or self.rot_fn is None:
            subs = self.cache.setdefault("subgraphs", {})
            if i not in subs:
                subs[i] = self.sub(*self.chunks[i])
            return subs[i]
        return self.sub(*self.chunks[i])

    def sub(self, e0, e1, n0, n1):
        """Edges [e0, e1) = every edge into nodes [n0, n1) (edges are dst-sorted).  Gathers
        still index all (extended) node rows; the node-path output covers rows [n0, n1)."""
        E = e1 - e0
        rot = self.rot[e0:e1] if self.rot is not None else self.rot_fn(e0, e1)
        g = Graph(self.src[e0:e1], self.dst[e0:e1], rot, (self.dst_ptr - e0).clamp(0, E),
                  self.num_nodes, self.lmax, self.mmax, None)
        g.num_nodes_ext = getattr(self, "num_nodes_ext", None) or self.num_nodes
        g.out_ptr = (self.dst_ptr[n0:n1 + 1] - e0).contiguous()
        g.dst_out = g.dst - n0
        g.num_out = n1 - n0
        return g


def chunk_bounds(dst_ptr, max_edges):
    """Split dst-sorted edges into chunks of whole destination nodes with at most ~max_edges
    edges (a node with more edges gets a chunk of its own): [(e0, e1, n0, n1)]."""
    import numpy as np

    ptr = np.asarray(dst_ptr)
    n = len(ptr) - 1
    out, n0 = [], 0
    while n0 < n:
        n1 = int(np.searchsorted(ptr, ptr[n0] + max_edges, side="right")) - 1
        n1 = min(max(n1, n0 + 1), n)
        out.append((int(ptr[n0]), int(ptr[n1]), n0, n1))
        n0 = n1
    return out


class eSEN_Backbone(nn.Module):
    """Atom embedding, edge-degree embedding, N x (node block [+ edge block]), final norm.

    Reference ``helm/esen_osh.py:57-485``.  ``forward`` takes a :class:`GraphBatch`
    (``maloq_b200.data.batch``) and returns the dict of the reference.
    """

    def __init__(self, irreps_out=None, max_num_elements=100, sphere_channels=128, lmax=2, mmax=2, cutoff=10.0,
                 edge_channels=128, distance_function="gaussian", num_distance_basis=512, num_layers=2,
                 hidden_channels=128, norm_type="rms_norm_sh", act_type="gate", mlp_type="spectral",
                 gaussian_width=1.0, include_edges=True, open_shell=False, wigner_backend="cuda",
                 distributed_graph_training=False, message_type="source-target", activation_checkpointing=False,
                 edge_chunk=None, edge_stream_dtype=torch.bfloat16, **unused):
        super().__init__()
        # recompute each block's forward during backward (saves only the block inputs); needed
        # for graphs whose per-layer edge activations exceed device memory
        self.activation_checkpointing = bool(activation_checkpointing)
        # graphs with more than edge_chunk edges run every block over chunks of whole
        # destination nodes (recomputed per chunk in backward) and keep the edge stream in bf16
        self.edge_chunk = int(edge_chunk) if edge_chunk else None
        self.edge_stream_dtype = edge_stream_dtype
        if act_type != "gate" or mlp_type != "spectral":
            raise ValueError("only act_type='gate' and mlp_type='spectral' are implemented (as in the reference)")
        self.max_num_elements, self.lmax, self.mmax = max_num_elements, lmax, mmax
        self.sphere_channels, self.hidden_channels = sphere_channels, hidden_channels
        self.include_edges, self.num_layers = include_edges, num_layers
        self.num_spins = 2 if open_shell else 1
        self.message_type = message_type
        for l, J in enumerate(sph.J_matrices(lmax, dtype=torch.float64)):
            self.register_buffer(f"Jd_{l}", J)
        self.sph_feature_size = (lmax + 1) ** 2
        self.mappingReduced = CoefficientMapping(lmax, mmax)
        self.sphere_embedding = nn.Embedding(max_num_elements, sphere_channels)
        self.abs_max_charge = 10
        self.charge_embedding = nn.Embedding(2 * self.abs_max_charge + 1, sphere_channels)
        self.max_spin_multiplicity = 11
        self.spin_embedding = nn.Embedding(self.max_spin_multiplicity, sphere_channels)
        self.scalar_node_embedding = nn.Linear(3 * sphere_channels, sphere_channels)
        self.cutoff, self.edge_channels, self.num_distance_basis = cutoff, edge_channels, num_distance_basis
        if distance_function == "gaussian":
            self.distance_expansion = GaussianSmearing(0.0, cutoff, num_distance_basis, gaussian_width)
        elif distance_function == "bessel":
            self.distance_expansion = EnvelopedBesselBasis(num_distance_basis, cutoff)
        else:
            raise ValueError("unknown distance function")
        self.source_embedding = nn.Embedding(max_num_elements, edge_channels)
        self.target_embedding = nn.Embedding(max_num_elements, edge_channels)
        nn.init.uniform_(self.source_embedding.weight.data, -0.001, 0.001)
        nn.init.uniform_(self.target_embedding.weight.data, -0.001, 0.001)
        self.edge_channels_list = [num_distance_basis + 2 * edge_channels, edge_channels, edge_channels]
        self.edge_degree_embedding = EdgeDegreeEmbedding(sphere_channels, lmax, mmax, self.edge_channels_list, 5.0,
                                                         self.mappingReduced)
        self.node_blocks = nn.ModuleList()
        if include_edges:
            self.edge_blocks = nn.ModuleList()
        for _ in range(num_layers):
            self.node_blocks.append(eSEN_Block(sphere_channels, hidden_channels, lmax, mmax, self.mappingReduced,
                                               self.edge_channels_list, norm_type, message_type, "node"))
            if include_edges:
                self.edge_blocks.append(eSEN_Block(sphere_channels, hidden_channels, lmax, mmax, self.mappingReduced,
                                                   self.edge_channels_list, norm_type, message_type, "edge"))
        self.norm = get_normalization_layer(norm_type, lmax, sphere_channels)

    # ---------------------------------------------------------------------------------
    def _rotations(self, edge_attr):
        vec = _model_frame(edge_attr)
        return ops.edge_rotation(vec, self.lmax, self.mmax, [getattr(self, f"Jd_{l}") for l in range(self.lmax + 1)],
                                 self.mappingReduced)

    def build_graph(self, batch) -> Graph:
        chunked = bool(self.edge_chunk and batch.num_edges > self.edge_chunk)
        # chunked inference computes each chunk's rotations on use instead of holding them all
        lazy_rot = chunked and not torch.is_grad_enabled()
        rot = None if lazy_rot else self._rotations(batch.edge_attr)
        g = Graph(batch.edge_index[0], batch.edge_index[1], rot, batch.dst_ptr, batch.num_nodes,
                  self.lmax, self.mmax, getattr(batch, "halo", None))
        g.num_nodes_ext = getattr(batch, "num_nodes_ext", None) or batch.num_nodes
        if chunked:
            host = getattr(batch, "dst_ptr_host", None)  # avoids reading dst_ptr back from the device
            g.chunks = chunk_bounds(host if host is not None else batch.dst_ptr.cpu().numpy(), self.edge_chunk)
            if lazy_rot:
                g.rot_fn = lambda e0, e1: self._rotations(batch.edge_attr[e0:e1])
        return g

    def forward(self, batch):
        graph = self.build_graph(batch)
        dist = batch.edge_attr[:, 0]
        z = batch.atomic_numbers
        n_local = graph.num_nodes
        z_local = z if getattr(batch, "local_node_ids", None) is None else z[batch.local_node_ids]
        charge = batch.atom_charge + self.abs_max_charge
        spin = batch.atom_spin
        emb = torch.cat([ops.embedding(z_local, self.sphere_embedding.weight),
                         ops.embedding(charge, self.charge_embedding.weight),
                         ops.embedding(spin, self.spin_embedding.weight)], -1)
        l0 = ops.linear(emb, self.scalar_node_embedding.weight, self.scalar_node_embedding.bias)
        x_node = l0.new_zeros(n_local, self.sph_feature_size, self.sphere_channels)
        x_node[:, 0] = l0
        if graph.chunks is None:
            # the radial MLPs' input: read by every block's radial MLP, only through GEMMs
            if isinstance(self.distance_expansion, GaussianSmearing):
                de = self.distance_expansion
                x_edge = ops.edge_inputs(batch.src_z, batch.dst_z, batch.edge_attr, self.source_embedding.weight,
                                         self.target_embedding.weight, de.offset, de.coeff)
            else:
                gauss = self.distance_expansion(dist)
                x_edge = ops.gemm_operand(torch.cat([ops.embedding(batch.src_z, self.source_embedding.weight), gauss,
                                                     ops.embedding(batch.dst_z, self.target_embedding.weight)], dim=1))
            x_node = self.edge_degree_embedding(x_node, x_edge, graph, "node")
            x_edge_emb = self.edge_degree_embedding(x_node, x_edge, graph, "edge") if self.include_edges else None
        else:
            x_edge = EdgeInputs(self, batch, dist)
            x_node, x_edge_emb = self._degree_embedding_chunked(x_node, x_edge, graph)
        ckpt = self.activation_checkpointing and torch.is_grad_enabled() and graph.chunks is None
        for i in range(self.num_layers):
            x_node = self._run_block(self.node_blocks[i], ckpt, x_node, x_edge_emb, x_edge, graph)
            if self.include_edges:
                x_edge_emb = self._run_block(self.edge_blocks[i], ckpt, x_node, x_edge_emb, x_edge, graph)
        x_node = self.norm(x_node)
        out = {"node_embeddings": x_node, "edge_index": batch.edge_index, "edge_distance": dist,
               "edge_distance_vec": _model_frame(batch.edge_attr), "partition": getattr(batch, "halo", None)}
        if self.include_edges and graph.chunks is not None:
            cd = x_node.dtype
            if torch.is_grad_enabled():
                out["edge_embeddings"] = torch.cat(
                    [_checkpointed(self._norm_rows, x_edge_emb[e0:e1], cd) for e0, e1, _, _ in graph.chunks], 0)
            else:  # in place on the edge stream
                for e0, e1, _, _ in graph.chunks:
                    x_edge_emb[e0:e1] = self._norm_rows(x_edge_emb[e0:e1], cd)
                out["edge_embeddings"] = x_edge_emb
            out["edge_chunks"] = [(e0, e1) for e0, e1, _, _ in graph.chunks]
        elif self.include_edges:
            out["edge_embeddings"] = self.norm(x_edge_emb)
        # edge features and graph for heads that run their own message pass (energy / force)
        out.update({"x_edge": x_edge, "graph": graph})
        return out

    def _degree_embedding_chunked(self, x_node, x_edge, graph):
        """Edge-degree embedding over the edge chunks: node rows of each chunk's destination
        range (base + scaled sum), and the edge stream (stored as ``edge_stream_dtype``)."""
        grad = torch.is_grad_enabled()
        run = _checkpointed if grad else (lambda f, *a: f(*a))
        ede = self.edge_degree_embedding

        def node_rows(base, e0, e1, sub):
            return ede(base, x_edge[e0:e1], sub, "node")

        def edge_rows(e0, e1, sub):
            return ede(None, x_edge[e0:e1], sub, "edge").to(self.edge_stream_dtype)

        parts = [run(node_rows, x_node[n0:n1], e0, e1, graph.chunk_graph(i))
                 for i, (e0, e1, n0, n1) in enumerate(graph.chunks)]
        x_node = torch.cat(parts, 0)
        if not self.include_edges:
            return x_node, None
        E = graph.src.shape[0]
        if grad:
            x_edge_emb = torch.cat([run(edge_rows, e0, e1, graph.chunk_graph(i))
                                    for i, (e0, e1, _, _) in enumerate(graph.chunks)], 0)
        else:
            x_edge_emb = torch.empty(E, self.sph_feature_size, self.sphere_channels, device=x_node.device,
                                     dtype=self.edge_stream_dtype)
            for i, (e0, e1, _, _) in enumerate(graph.chunks):
                x_edge_emb[e0:e1] = edge_rows(e0, e1, graph.chunk_graph(i))
        return x_node, x_edge_emb

    def _norm_rows(self, x, compute_dtype):
        return self.norm(x.to(compute_dtype)).to(x.dtype)

    @staticmethod
    def _run_block(block, ckpt, x_node, x_edge_emb, x_edge, graph):
        if not ckpt:
            return block(x_node, x_edge_emb, x_edge, graph)
        from torch.utils.checkpoint import checkpoint

        return checkpoint(block, x_node, x_edge_emb, x_edge, graph, use_reentrant=False)

    @property
    def num_params(self):
        return sum(p.numel() for p in self.parameters())

    def no_weight_decay(self) -> set:
        """Biases, norm affine parameters and LayerNorm parameters (``esen_osh.py:492-517``)."""
        out = set()
        for name, _ in self.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            if leaf in ("bias", "affine_weight", "affine_bias") or ".net.1." in name or ".net.4." in name:
                out.add(name)
        return out
