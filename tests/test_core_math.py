"""Spherical harmonics, Wigner-D, J matrices, Wigner 3j and the basis transform."""
import numpy as np
import pytest
import torch

from maloq_b200.core import sph, wigner3j
from maloq_b200.core.irreps import Irreps, make_label_layout, sorted_to_original_permutation
from maloq_b200.data import basis_sets


def _rand_rot(rng):
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    a, b, c, d = q
    return np.array([[a*a+b*b-c*c-d*d, 2*(b*c-a*d), 2*(b*d+a*c)],
                     [2*(b*c+a*d), a*a-b*b+c*c-d*d, 2*(c*d-a*b)],
                     [2*(b*d-a*c), 2*(c*d+a*b), a*a-b*b-c*c+d*d]])


@pytest.mark.parametrize("l", range(0, 9))
def test_wigner_D_orthogonal_and_homomorphism(l):
    rng = np.random.default_rng(l)
    R1, R2 = _rand_rot(rng), _rand_rot(rng)
    D1, D2 = sph.wigner_D_from_matrix(l, R1), sph.wigner_D_from_matrix(l, R2)
    np.testing.assert_allclose(D1 @ D1.T, np.eye(2 * l + 1), atol=1e-10)
    np.testing.assert_allclose(sph.wigner_D_from_matrix(l, R1 @ R2), D1 @ D2, atol=1e-10)


@pytest.mark.parametrize("l", range(0, 7))
def test_euler_formula_matches_matrix(l):
    a, b, g = 0.3, 1.1, -0.7
    J = torch.tensor(sph.J_matrix(l))
    D = sph.wigner_D(l, torch.tensor(a, dtype=torch.float64), torch.tensor(b, dtype=torch.float64),
                     torch.tensor(g, dtype=torch.float64), J).numpy()
    np.testing.assert_allclose(D, sph.wigner_D_from_matrix(l, sph.euler_matrix(a, b, g)), atol=1e-12)


def test_J_is_involution_and_l1_is_xy_swap():
    np.testing.assert_allclose(sph.J_matrix(1), [[0, -1, 0], [-1, 0, 0], [0, 0, 1]], atol=1e-14)
    for l in range(12):
        J = sph.J_matrix(l)
        np.testing.assert_allclose(J @ J, np.eye(2 * l + 1), atol=1e-12)


def test_edge_rotation_aligns_edge_with_polar_axis():
    rng = np.random.default_rng(0)
    v = torch.tensor(rng.normal(size=(50, 3)))
    alpha, beta = sph.edge_euler_angles(v)
    J1 = torch.tensor(sph.J_matrix(1))
    D = sph.wigner_D(1, torch.zeros_like(alpha), -beta, -alpha, J1)  # [E, 3, 3] on (x, y, z)
    u = torch.nn.functional.normalize(v, dim=-1)
    r = torch.einsum("eij,ej->ei", D, u)
    np.testing.assert_allclose(r.numpy(), np.tile([0.0, 1.0, 0.0], (50, 1)), atol=1e-10)


@pytest.mark.parametrize("ls", [(1, 1, 0), (1, 1, 1), (1, 2, 3), (2, 2, 2), (3, 2, 4), (0, 3, 3)])
def test_wigner3j_invariant_and_normalised(ls):
    l1, l2, l3 = ls
    C = wigner3j._wigner_3j_np(l1, l2, l3)
    assert abs(np.linalg.norm(C) - 1) < 1e-12
    R = _rand_rot(np.random.default_rng(7))
    D1, D2, D3 = (sph.wigner_D_from_matrix(l, R) for l in ls)
    C2 = np.einsum("ia,jb,kc,abc->ijk", D1, D2, D3, C)
    np.testing.assert_allclose(C2, C, atol=1e-10)


def test_basis_transform_roundtrip_and_equivariance():
    layout = make_label_layout(basis_sets.get_basis("def2_svp_like"))
    bt = wigner3j.BasisTransform(layout.out_js_list, dtype=torch.float64)
    D = layout.target_len
    x = torch.randn(7, D, dtype=torch.float64)
    np.testing.assert_allclose(bt.get_net_out(bt.get_H(x)).numpy(), x.numpy(), atol=1e-10)
    # coupled components of an (l1, l2) block rotate as irreps l3 when the block rotates as D1 H D2^T
    R = _rand_rot(np.random.default_rng(3))
    h = bt.get_H(x)
    hr = h.clone()
    for (l1, l2), s in zip(layout.out_js_list, bt.H_slices[:-1]):
        a, b = l1 % 10, l2 % 10
        n1, n2 = 2 * a + 1, 2 * b + 1
        blk = h[:, s:s + n1 * n2].reshape(-1, n1, n2)
        D1, D2 = (torch.tensor(sph.wigner_D_from_matrix(l, R)) for l in (a, b))
        hr[:, s:s + n1 * n2] = (D1 @ blk @ D2.T).reshape(-1, n1 * n2)
    xr = bt.get_net_out(hr)
    exp = x.clone()
    for it, (s0, s1) in zip(layout.irreps_out, layout.irreps_out.slices()):
        Dl = torch.tensor(sph.wigner_D_from_matrix(it.l, R))
        exp[:, s0:s1] = x[:, s0:s1] @ Dl.T
    np.testing.assert_allclose(xr.numpy(), exp.numpy(), atol=1e-9)


def test_irreps_sort_permutation():
    irr = Irreps("1x2e+1x0e+1x1e+1x0e")
    srt, p, inv = irr.sort()
    assert str(srt) == "1x0e+1x0e+1x1e+1x2e"
    perm = sorted_to_original_permutation(irr)
    sorted_vals = torch.arange(srt.dim)
    orig = sorted_vals[perm]
    # sorted: 0e(#1) 0e(#3) 1e(#2) 2e(#0) -> original order 2e, 0e, 1e, 0e
    assert orig.tolist() == [5, 6, 7, 8, 9, 0, 2, 3, 4, 1]


def test_basis_transform_column_tables_and_transposes():
    """The per-column tables the row kernel uses reproduce x @ W, x @ W_inv and (for the
    backward) x @ W^T, x @ W_inv^T."""
    import numpy as np

    from maloq_b200.data import datasets

    T = datasets.labeler_for("druglike").transform
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, T.dim))
    for inverse in (False, True):
        W = (T.W_global_inv if inverse else T.W_global).double().numpy()
        for transpose, ref in ((False, x @ W), (True, x @ W.T)):
            meta, coef = T.column_tables(inverse, transpose)
            out = np.zeros_like(x)
            for u, (s, n, c, _) in enumerate(meta):
                out[:, u] = x[:, s:s + n] @ coef[c + np.arange(n) * n]
            assert np.allclose(out, ref, atol=1e-6)


# largest entry of wigner_3j(l1, l2, l3) for every triple of an s/p/d basis (def2-SVP-like
# layouts): the e3nn construction (Racah Clebsch-Gordan + real change of basis with the
# (-i)^l factor, unit norm) fixes each triple's sign; these values pin it
_W3J_PINS = {(0, 0, 0): ((0, 0, 0), 1.0), (0, 1, 1): ((0, 1, 1), 0.57735), (0, 2, 2): ((0, 2, 2), 0.447214),
             (1, 0, 1): ((1, 0, 1), 0.57735), (1, 1, 0): ((1, 1, 0), 0.57735), (1, 1, 1): ((0, 1, 2), 0.408248),
             (1, 1, 2): ((1, 1, 2), 0.365148), (1, 2, 1): ((1, 2, 1), 0.365148), (1, 2, 2): ((1, 0, 4), -0.365148),
             (1, 2, 3): ((1, 2, 3), 0.29277), (2, 0, 2): ((2, 0, 2), 0.447214), (2, 1, 1): ((2, 1, 1), 0.365148),
             (2, 1, 2): ((0, 1, 4), 0.365148), (2, 1, 3): ((2, 1, 3), 0.29277), (2, 2, 0): ((2, 2, 0), 0.447214),
             (2, 2, 1): ((0, 4, 1), -0.365148), (2, 2, 2): ((2, 2, 2), 0.239046), (2, 2, 3): ((0, 2, 5), 0.267261),
             (2, 2, 4): ((2, 2, 4), 0.239046)}


def test_wigner3j_signs_pinned_to_e3nn_construction():
    from maloq_b200.core import wigner3j

    for (l1, l2, l3), (idx, val) in _W3J_PINS.items():
        C = wigner3j.wigner_3j(l1, l2, l3, dtype=torch.float64)
        assert abs(C[idx].item() - val) < 1e-6, ((l1, l2, l3), C[idx].item(), val)
        # the pinned entry is the largest in magnitude (so the sign is unambiguous)
        assert abs(val) >= C.abs().max().item() - 1e-6
