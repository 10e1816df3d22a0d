"""Selectable model variants (CPU): the three equivariant norms and the degree layer scale,
SO2_Linear, the S^2 grid and grid activations, each against a direct restatement of its
definition and for rotation equivariance."""
import math

import numpy as np
import pytest
import torch

from maloq_b200.core import sph
from maloq_b200.models import layers


def _x(n=5, L=3, C=6, seed=0, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, (L + 1) ** 2, C, generator=g, dtype=dtype)


def _affine(norm, seed=1):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in norm.parameters():
            p.copy_(torch.randn(p.shape, generator=g, dtype=p.dtype))


def _layer_norm_loops(x, w, b, L, eps):
    out = []
    for l in range(L + 1):
        f = x[:, l * l:(l + 1) ** 2]
        if l == 0:
            f = f - f.mean(dim=2, keepdim=True)
        n = f.pow(2).mean(dim=1, keepdim=True).mean(dim=2, keepdim=True)
        f = f * ((n + eps) ** -0.5 * w[l].view(1, 1, -1))
        if l == 0:
            f = f + b.view(1, 1, -1)
        out.append(f)
    return torch.cat(out, 1)


def _layer_norm_sh_loops(x, ln, w, L, eps):
    out = [ln(x[:, :1])]
    f = x[:, 1:]
    n = torch.zeros(x.shape[0], 1, x.shape[2], dtype=x.dtype)
    for l in range(1, L + 1):
        n = n + f[:, l * l - 1:(l + 1) ** 2 - 1].pow(2).sum(1, keepdim=True) / (2 * l + 1) / L
    s = (n.mean(dim=2, keepdim=True) + eps) ** -0.5
    for l in range(1, L + 1):
        out.append(x[:, l * l:(l + 1) ** 2] * s * w[l - 1].view(1, 1, -1))
    return torch.cat(out, 1)


def test_layer_norms_match_definitions():
    L, C = 3, 6
    x = _x(L=L, C=C)
    n1 = layers.get_normalization_layer("layer_norm", L, C).double()
    _affine(n1)
    ref = _layer_norm_loops(x, n1.affine_weight, n1.affine_bias, L, n1.eps)
    assert torch.allclose(n1(x), ref, atol=1e-12)
    n2 = layers.get_normalization_layer("layer_norm_sh", L, C).double()
    _affine(n2)
    ref2 = _layer_norm_sh_loops(x, n2.norm_l0, n2.affine_weight, L, n2.eps)
    assert torch.allclose(n2(x), ref2, atol=1e-12)
    # residual convention shared with rms_norm_sh
    r = _x(L=L, C=C, seed=3)
    y, s = n2(x, residual=r)
    assert torch.allclose(s, x + r) and torch.allclose(y, n2(x + r))
    with pytest.raises(ValueError):
        layers.get_normalization_layer("batch_norm", L, C)


def test_degree_layer_scale():
    L, C = 3, 4
    ls = layers.EquivariantDegreeLayerScale(L, C).double()
    x = _x(L=L, C=C)
    y = ls(x)
    for l in range(L + 1):
        f = 1.0 if l == 0 else 1 / math.sqrt(2.0 * l)
        assert torch.allclose(y[:, l * l:(l + 1) ** 2], x[:, l * l:(l + 1) ** 2] * f)


def _D(L, R):
    return torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(l, R)) for l in range(L + 1)])


@pytest.mark.parametrize("norm_type", ["layer_norm", "layer_norm_sh", "rms_norm_sh"])
def test_norms_equivariant(norm_type):
    L, C = 4, 5
    norm = layers.get_normalization_layer(norm_type, L, C).double()
    _affine(norm)
    x = _x(L=L, C=C)
    D = _D(L, sph.euler_matrix(0.3, 1.1, -0.7))
    a = torch.einsum("ij,njc->nic", D, norm(x))
    b = norm(torch.einsum("ij,njc->nic", D, x))
    assert (a - b).abs().max().item() < 1e-10


@pytest.mark.parametrize("norm_type", ["layer_norm", "layer_norm_sh"])
def test_backbone_with_norm_type_equivariant(norm_type):
    from maloq_b200.data import basis_sets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.models.backbone import eSEN_Backbone

    lab = FockLabeler(basis_sets.get_basis("split_valence_small"), dtype=torch.float64)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=5.0, num_layers=2,
                       num_distance_basis=8, edge_channels=8, norm_type=norm_type).double()
    rng = np.random.default_rng(1)
    structs = [structures.random_small_molecule(rng) for _ in range(2)]
    P = np.array([[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])
    R_in = sph.euler_matrix(0.4, -1.2, 2.0)
    b0 = collate([make_sample(s, 5.0) for s in structs], lab.table, float_dtype=torch.float64)
    b1 = collate([make_sample(structures.Structure(s.z, s.pos @ R_in.T), 5.0) for s in structs], lab.table,
                 float_dtype=torch.float64)
    e0, e1 = bb(b0), bb(b1)
    D = _D(4, P @ R_in @ P.T)
    for key in ("node_embeddings", "edge_embeddings"):
        err = (torch.einsum("ij,njc->nic", D, e0[key]) - e1[key]).abs().max().item()
        assert err < 1e-9, (key, err)


def _rot_about_polar(g):
    # rotation about the y (polar) axis of the harmonic basis
    c, s = math.cos(g), math.sin(g)
    return np.array([[c, 0.0, s], [0.0, 1.0, 0.0], [-s, 0.0, c]])


@pytest.mark.parametrize("mmax", [2, 3])
def test_so2_linear_commutes_with_rolls(mmax):
    L, C = 3, 4
    torch.manual_seed(2)
    lin = layers.SO2_Linear(C, 5, L, mmax, edge_channels_list=[6, 8]).double()
    x = _x(n=7, L=L, C=C)
    # zero the |m| > mmax entries (the layer ignores them)
    keep = torch.zeros((L + 1) ** 2, dtype=torch.bool)
    keep[lin.mapping.m_to_lm] = True
    x = x * keep.view(1, -1, 1)
    xe = torch.randn(7, 6, dtype=torch.float64)
    y = lin(x, xe)
    assert y.shape == (7, (L + 1) ** 2, 5) and (y[:, ~keep] == 0).all()
    D = _D(L, _rot_about_polar(0.77))
    a = torch.einsum("ij,njc->nic", D, y)
    b = lin(torch.einsum("ij,njc->nic", D, x), xe)
    assert (a - b).abs().max().item() < 1e-10
    # m = 0 path equals a direct linear on the m = 0 entries times the radial weights
    rad = lin.rad_func(xe)
    m0 = [l * l + l for l in range(L + 1)]
    x0 = x[:, m0].reshape(7, -1) * rad[:, : (L + 1) * C]
    assert torch.allclose(y[:, m0], lin.fc_m0(x0).view(7, L + 1, 5))


@pytest.mark.parametrize("lmax,mmax,norm", [(3, 3, "integral"), (4, 2, "integral"), (3, 3, "component")])
def test_so3_grid_round_trip(lmax, mmax, norm):
    grid = layers.SO3_Grid(lmax, mmax, normalization=norm, rescale=False)
    n_coef = grid.to_grid_mat.shape[-1]
    assert n_coef == sum(min(2 * l + 1, 2 * mmax + 1) for l in range(lmax + 1))
    x = torch.randn(3, n_coef, 4)
    back = grid.from_grid(grid.to_grid(x))
    assert torch.allclose(back, x, atol=1e-5)


def test_s2_activation():
    L = 3
    grid = layers.SO3_Grid(L, L, resolution=24)
    act = layers.S2Activation(L, L, {"lmax_mmax": grid})
    x = torch.zeros(2, (L + 1) ** 2, 3)
    x[:, 0] = torch.randn(2, 3)
    # a constant function on the sphere stays constant: only l = 0 survives, silu applied to its value
    y = act(x)
    y00 = math.sqrt(1 / (4 * math.pi))
    val = x[:, 0] * y00
    assert torch.allclose(y[:, 0] * y00, torch.nn.functional.silu(val), atol=1e-5)
    assert y[:, 1:].abs().max() < 1e-5
    sep = layers.SeparableS2Activation(L, L, grid)
    s = torch.randn(2, 3)
    z = sep(s, torch.randn(2, (L + 1) ** 2, 3))
    assert torch.allclose(z[:, 0], torch.nn.functional.silu(s))
