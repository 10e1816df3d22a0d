"""Hamiltonian-MAE parity of the kernel path on the GPU: the same training run (fixed synthetic
Fock targets, same initial weights) on the PyTorch ops in fp32 and on the sm_100a kernels with
bf16 GEMM operands ends at the same Hamiltonian MAE within 10 %."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _train_mae(steps, dev, torch_ops):
    from maloq_b200 import ops
    from maloq_b200.data import datasets
    from maloq_b200.data.batch import collate
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    lab = datasets.labeler_for("druglike")
    kw = dict(sphere_channels=64, hidden_channels=64, lmax=lab.layout.lmax, mmax=2, cutoff=6.0, num_layers=2,
              num_distance_basis=32, edge_channels=64)
    samples, _ = datasets.build_dataset("druglike", 4, kw, seed=3, labeler=lab)
    b = collate(samples, lab.table).to(dev)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, include_edges=True, **kw).to(dev)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=lab.layout.lmax, sphere_channels=64, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True).to(dev)
    ops.use_torch_ops(torch_ops)
    try:
        opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()), lr=2e-3)
        tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask))
        for _ in range(steps):
            tr.train_step(b, L.rmse_mse_padded_loss, opt)
        with torch.no_grad():
            no, eo = hd(bb(b), b)
    finally:
        ops.use_torch_ops(False)
    no, eo = no[0].float().cpu(), eo[0].float().cpu()
    maes, n0, e0 = [], 0, 0
    for s in samples:
        n1, e1 = n0 + s.num_nodes, e0 + s.num_edges
        Hp = lab.blocks_from_labels(s, no[n0:n1].to(lab.device), eo[e0:e1].to(lab.device)).to_dense()
        Ht = lab.blocks_from_labels(s, s.node_y[0].to(lab.device), s.y[0].to(lab.device)).to_dense()
        maes.append(float(np.abs(Hp - Ht).mean()))
        n0, e0 = n1, e1
    return float(np.mean(maes))


def test_trained_hamiltonian_mae_kernel_path_matches_fp32_pytorch(cuda_device):
    from maloq_b200.ops import kernels

    mae0 = _train_mae(0, cuda_device, True)
    ref = _train_mae(30, cuda_device, True)
    got = _train_mae(30, cuda_device, False)
    print(f"Hamiltonian MAE: untrained {mae0:.4g}, fp32 PyTorch ops {ref:.4g}, bf16 kernels {got:.4g}")
    assert ref < 0.8 * mae0
    assert abs(got - ref) <= 0.1 * ref, (ref, got)
    assert kernels.error_status() == 0


@pytest.mark.parametrize("kind", ["energies", "forces"])
def test_energy_and_force_heads_kernel_path(cuda_device, kind):
    """Energy / force heads on the kernel path (their convolution has C or one output channel,
    padded to 8 for the kernels) against the fp32 PyTorch ops: loss and head gradients."""
    from maloq_b200 import ops
    from maloq_b200.data import datasets
    from maloq_b200.data.batch import collate
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import HELM_Energy_Head, HELM_Force_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    lab = datasets.labeler_for("small")
    kw = dict(sphere_channels=32, hidden_channels=32, lmax=4, mmax=2, cutoff=5.0, num_layers=1,
              num_distance_basis=16, edge_channels=32)
    samples = datasets.build_samples("small", 6, seed=1)
    b = collate(samples, lab.table).to(cuda_device)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, include_edges=False, **kw).to(cuda_device)
    hd = (HELM_Energy_Head if kind == "energies" else HELM_Force_Head)(bb).to(cuda_device)
    # zero targets: the loss's relative error is then the prediction's
    if kind == "energies":
        b.energy = torch.zeros(b.num_graphs, device=cuda_device)
    else:
        b.forces = torch.zeros(b.num_nodes, 3, device=cuda_device)

    def step(torch_ops):
        ops.use_torch_ops(torch_ops)
        try:
            tr = SplitTrainer(bb, hd, lab.irreps)
            for p in list(bb.parameters()) + list(hd.parameters()):
                p.grad = None
            _, _, loss = tr.forward_loss(b, L.mse_padded_loss)
            loss.backward()
        finally:
            ops.use_torch_ops(False)
        return float(loss.detach()), {n: p.grad.clone() for n, p in hd.named_parameters() if p.grad is not None}

    ref, got = step(True), step(False)
    assert abs(got[0] - ref[0]) <= 2e-2 * abs(ref[0])
    for n, g in ref[1].items():
        assert ((got[1][n] - g).norm() / (g.norm() + 1e-12)).item() < 5e-2, n
