"""Rotation-equivariance error of the backbone + Fock head.

The model is run on a batch of molecules and on the same molecules rotated by a random
rotation R; the Hamiltonian labels must transform with the block-diagonal Wigner matrix of
the label irreps (the node and edge blocks rotate like the orbitals they couple).  The error is
``max |D y(x) - y(R x)| / max |y(x)|`` over the node and edge outputs.  Input coordinates are
(x, y, z); the model's harmonic frame is (y, z, x).
"""

from __future__ import annotations

import numpy as np
import torch


def random_rotation(rng) -> np.ndarray:
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    a, b, c, d = q
    return np.array([[a * a + b * b - c * c - d * d, 2 * (b * c - a * d), 2 * (b * d + a * c)],
                     [2 * (b * c + a * d), a * a - b * b + c * c - d * d, 2 * (c * d - a * b)],
                     [2 * (b * d - a * c), 2 * (c * d + a * b), a * a - b * b - c * c + d * d]])


def model_equivariance_error(backbone, head, structures_, labeler, cutoff, R, device) -> float:
    """Relative equivariance error of ``head(backbone(.))`` under the rotation ``R``."""
    from ..core import sph
    from ..data import structures as S
    from ..data.batch import collate, make_sample

    P = np.array([[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])
    b0 = collate([make_sample(s, cutoff) for s in structures_], labeler.table).to(device)
    b1 = collate([make_sample(S.Structure(s.z, s.pos @ R.T), cutoff) for s in structures_], labeler.table).to(device)
    with torch.no_grad():
        n0, e0 = head(backbone(b0), b0)
        n1, e1 = head(backbone(b1), b1)
    D = torch.block_diag(*[torch.tensor(sph.wigner_D_from_matrix(it.l, P @ R @ P.T), dtype=torch.float32)
                           for it in labeler.irreps]).to(device)
    scale = max(n0.abs().max().item(), e0.abs().max().item(), 1e-12)
    err = max((n0[0].float() @ D.T - n1[0].float()).abs().max().item(),
              (e0[0].float() @ D.T - e1[0].float()).abs().max().item())
    return err / scale


def rotation_equivariance_error(device, seed=0, channels=32, layers=2, n_mol=3) -> float:
    """Equivariance error of a random-init drug-like model (lmax 4, mmax 2, def2-SVP-like
    labels) on ``n_mol`` random drug-like molecules of 12-20 atoms."""
    from ..data import basis_sets, structures
    from ..data.targets import FockLabeler
    from ..models.backbone import eSEN_Backbone
    from ..models.heads import Fock_Irreps_Head

    torch.manual_seed(seed)
    rng = np.random.default_rng(seed)
    lab = FockLabeler(basis_sets.get_basis("def2_svp_like"), device=device)
    bb = eSEN_Backbone(lab.irreps, sphere_channels=channels, hidden_channels=channels, lmax=4, mmax=2, cutoff=6.0,
                       edge_channels=channels, num_layers=layers, num_distance_basis=16).to(device)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=channels, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True).to(device)
    mols = [structures.random_druglike_molecule(rng, 12, 20) for _ in range(n_mol)]
    return model_equivariance_error(bb, hd, mols, lab, 6.0, random_rotation(rng), device)
