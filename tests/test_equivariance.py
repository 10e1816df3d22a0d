"""Hard-asserted rotation equivariance of the backbone and the Fock head (fp64, CPU).

The reference only plots these errors (tests/test_equivariance.py:152-188); here the
rotated-input outputs must equal the rotated outputs to 1e-9 (fp64) / 1e-5 (fp32).
"""
import numpy as np
import pytest
import torch

from maloq_b200.core import sph
from maloq_b200.data import basis_sets, structures
from maloq_b200.data.batch import collate, make_sample
from maloq_b200.data.targets import FockLabeler
from maloq_b200.models.backbone import eSEN_Backbone
from maloq_b200.models.heads import Fock_Irreps_Head

P = np.array([[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])  # input (x,y,z) -> model (y,z,x)


def _rot(seed):
    rng = np.random.default_rng(seed)
    a, b, g = rng.uniform(-np.pi, np.pi, 3)
    return sph.euler_matrix(a, b, g)


def _block_D(lmax, R):
    return torch.tensor(sph.rotation_to_wigner_numeric(lmax, R))


def _models(lab, dtype, mmax=2, message_type="source-target", reduce=True):
    torch.manual_seed(0)
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=mmax, cutoff=5.0, num_layers=2,
              num_distance_basis=8, edge_channels=8, message_type=message_type)
    bb = eSEN_Backbone(lab.irreps, **kw).to(dtype)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list,
                          reduce_node=reduce, reduce_node_intra=reduce).to(dtype)
    return bb, hd


def _batch(structs, lab, R_in, dtype):
    out = []
    for s in structs:
        s2 = structures.Structure(s.z, s.pos @ R_in.T)
        out.append(make_sample(s2, 5.0))
    return collate(out, lab.table, float_dtype=dtype)


@pytest.mark.parametrize("mmax,message_type,reduce", [(2, "source-target", True), (4, "source-target", False),
                                                       (2, "source-target-message", True)])
def test_backbone_and_head_equivariant_fp64(mmax, message_type, reduce):
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"), dtype=torch.float64)
    rng = np.random.default_rng(1)
    structs = [structures.random_small_molecule(rng) for _ in range(3)]
    bb, hd = _models(lab, torch.float64, mmax, message_type, reduce)
    R_in = _rot(5)
    R_model = P @ R_in @ P.T
    b0 = _batch(structs, lab, np.eye(3), torch.float64)
    b1 = _batch(structs, lab, R_in, torch.float64)
    # same graph (rotation keeps distances); edge order identical because sorting is by index
    assert torch.equal(b0.edge_index, b1.edge_index)
    e0, e1 = bb(b0), bb(b1)
    D = _block_D(4, R_model)
    for key in ("node_embeddings", "edge_embeddings"):
        rot = torch.einsum("ij,njc->nic", D, e0[key])
        err = (rot - e1[key]).abs().max().item()
        assert err < 1e-9, (key, err)
    n0, ed0 = hd(e0, b0)
    n1, ed1 = hd(e1, b1)
    Dl = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(it.l, R_model)) for it in lab.irreps])
    assert (n0[0] @ Dl.T - n1[0]).abs().max().item() < 1e-9
    assert (ed0[0] @ Dl.T - ed1[0]).abs().max().item() < 1e-9


def test_equivariance_fp32_within_1e5():
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    rng = np.random.default_rng(2)
    structs = [structures.random_small_molecule(rng) for _ in range(2)]
    bb, hd = _models(lab, torch.float32)
    R_in = _rot(9)
    R_model = P @ R_in @ P.T
    b0 = _batch(structs, lab, np.eye(3), torch.float32)
    b1 = _batch(structs, lab, R_in, torch.float32)
    n0, ed0 = hd(bb(b0), b0)
    n1, ed1 = hd(bb(b1), b1)
    Dl = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(it.l, R_model), dtype=torch.float32)
                            for it in lab.irreps])
    scale = max(n0.abs().max().item(), ed0.abs().max().item(), 1.0)
    assert (n0[0] @ Dl.T - n1[0]).abs().max().item() / scale < 1e-5
    assert (ed0[0] @ Dl.T - ed1[0]).abs().max().item() / scale < 1e-5
