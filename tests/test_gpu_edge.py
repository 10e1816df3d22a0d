"""Fused Edgewise kernels vs the fp32 PyTorch definition of the same op (forward + grads)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(dev, message_type, C=32, mmax=2, n_mol=3, seed=0):
    from maloq_b200.data import basis_sets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.models.backbone import eSEN_Backbone

    torch.manual_seed(seed)
    lab = FockLabeler(basis_sets.get_basis("def2_svp_like"))
    rng = np.random.default_rng(seed)
    samples = [make_sample(structures.random_druglike_molecule(rng, 12, 20), 6.0) for _ in range(n_mol)]
    b = collate(samples, lab.table).to(dev)
    bb = eSEN_Backbone(lab.irreps, sphere_channels=C, hidden_channels=C, lmax=4, mmax=mmax, cutoff=6.0,
                       edge_channels=C, num_layers=1, num_distance_basis=16, message_type=message_type).to(dev)
    return bb, b


def _rel(a, b):
    return ((a - b).abs().max() / (b.abs().max() + 1e-12)).item()


def _relf(a, b):
    """Relative Frobenius error (the typical, rather than worst, element error)."""
    return ((a - b).float().norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("path", ["node", "edge"])
@pytest.mark.parametrize("message_type,mmax", [("source-target", 2), ("source-target-message", 2),
                                               ("source-target", 4)])
def test_edgewise_matches_reference(cuda_device, path, message_type, mmax):
    from maloq_b200.ops import edge_native
    from maloq_b200.ops import reference as R

    bb, b = _setup(cuda_device, message_type, mmax=mmax)
    graph = bb.build_graph(b)
    mod = bb.node_blocks[0].edge_wise
    E, N, S, C = b.num_edges, b.num_nodes, 25, 32
    torch.manual_seed(1)
    x = torch.randn(N, S, C, device=cuda_device, requires_grad=True)
    xe = torch.randn(E, S, C, device=cuda_device, requires_grad=True) if message_type.endswith("message") else None
    x_edge = torch.randn(E, 2 * C + 16, device=cuda_device, requires_grad=True)
    out = edge_native.edgewise(mod, x, xe, x_edge, graph, path)
    gout = torch.randn_like(out)
    grads = torch.autograd.grad((out * gout).sum(), [x, x_edge] + ([xe] if xe is not None else []) +
                                list(mod.parameters()), allow_unused=True)
    ref = R.edgewise(mod, x, xe, x_edge, graph, path)
    rgrads = torch.autograd.grad((ref * gout).sum(), [x, x_edge] + ([xe] if xe is not None else []) +
                                 list(mod.parameters()), allow_unused=True)
    assert _rel(out, ref) < 2e-2
    assert _relf(out, ref) < 1e-2, _relf(out, ref)
    print(path, message_type, mmax, "out", _rel(out, ref), _relf(out, ref))
    names = ["x", "x_edge"] + (["xe"] if xe is not None else []) + [n for n, _ in mod.named_parameters()]
    for n, g, rg in zip(names, grads, rgrads):
        if rg is None:
            continue
        assert g is not None, n
        assert _rel(g, rg) < 3e-2, (n, _rel(g, rg))
        assert _relf(g, rg) < 1.5e-2, (n, _relf(g, rg))
        print("  grad", n, _rel(g, rg), _relf(g, rg))
    from maloq_b200.ops import kernels

    assert kernels.error_status() == 0


def test_edge_degree_embedding_matches_reference(cuda_device):
    from maloq_b200.ops import edge_native
    from maloq_b200.ops import reference as R

    bb, b = _setup(cuda_device, "source-target")
    graph = bb.build_graph(b)
    E, N, C = b.num_edges, b.num_nodes, 32
    e = torch.randn(E, 5, C, device=cuda_device, requires_grad=True)
    base = torch.randn(N, 25, C, device=cuda_device, requires_grad=True)
    out = edge_native.rotate_back_m0(e, graph, base=base, scale=0.2)
    ref = base + R.scatter_sum(R.rotate_back_m0(e, graph.rot) * 0.2, graph.dst, N)
    g = torch.randn_like(out)
    ge, gb = torch.autograd.grad((out * g).sum(), [e, base])
    re_, rb = torch.autograd.grad((ref * g).sum(), [e, base])
    assert _rel(out, ref) < 1e-2, _rel(out, ref)
    assert _rel(ge, re_) < 1e-4, _rel(ge, re_)
    assert _rel(gb, rb) < 1e-6, _rel(gb, rb)
    out2 = edge_native.rotate_back_m0(e, graph)
    assert _rel(out2, R.rotate_back_m0(e, graph.rot)) < 1e-2


def test_edgewise_deterministic(cuda_device):
    from maloq_b200.ops import edge_native

    bb, b = _setup(cuda_device, "source-target")
    graph = bb.build_graph(b)
    mod = bb.node_blocks[0].edge_wise
    x = torch.randn(b.num_nodes, 25, 32, device=cuda_device, requires_grad=True)
    x_edge = torch.randn(b.num_edges, 80, device=cuda_device)
    outs = []
    for _ in range(2):
        y = edge_native.edgewise(mod, x, None, x_edge, graph, "node")
        (g,) = torch.autograd.grad(y.square().sum(), [x])
        outs.append((y, g))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
