"""Multi-GPU tests (need >= 2 GPUs; skipped otherwise): fused NVLink all-reduce vs NCCL."""
import pytest
import torch

from tests import _dist_util

pytestmark = pytest.mark.gpu


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _allreduce_worker(rank, world, multimem):
    import torch
    import torch.distributed as dist

    from maloq_b200.ops import kernels
    from maloq_b200.parallel.symm import PeerAllReduce

    dev = torch.device("cuda", rank)
    par = PeerAllReduce(1 << 20, dev, use_multimem=multimem)
    res = []
    for trial in range(3):
        n = [1000003 - 4, 4096, 12345 * 4][trial]
        torch.manual_seed(trial * 10 + rank)
        x = torch.randn(n, device=dev)
        v = par.view(16 * trial, n)
        v.copy_(x)
        par.all_reduce_(v, side_stream=None, scale=1.0 / world)
        par.wait(torch.cuda.current_stream(dev))
        ref = x.clone()
        dist.all_reduce(ref)
        ref /= world
        res.append((v - ref).abs().max().item())
    torch.cuda.synchronize()
    return res, par.transport, kernels.error_status()


@pytest.mark.parametrize("multimem", [False, None])
def test_peer_allreduce_matches_nccl(multimem):
    _need(2)
    out = _dist_util.run(_allreduce_worker, world=2, backend="nccl", args=(multimem,))
    for r, (errs, transport, status) in out.items():
        assert status == 0, status
        assert max(errs) < 1e-5, (transport, errs)


def _train_worker(rank, world):
    import torch

    from maloq_b200.data import batch as B
    from maloq_b200.data import datasets
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.parallel.dp import GradSync
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    dev = torch.device("cuda", rank)
    lab = datasets.labeler_for("druglike", dev)
    kw = dict(sphere_channels=32, hidden_channels=32, lmax=4, mmax=2, cutoff=6.0, edge_channels=32, num_layers=2,
              num_distance_basis=16)
    samples, _ = datasets.build_dataset("druglike", 4, kw, seed=rank, device=dev, labeler=lab)
    batch = B.collate(samples, lab.table).to(dev)
    grads = {}
    for mode in ("nccl", "fused"):
        torch.manual_seed(5)
        bb = eSEN_Backbone(lab.irreps, **kw).to(dev)
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=32, ls_list=lab.layout.ls_list,
                              reduce_node=True, reduce_node_intra=True).to(dev)
        params = list(bb.parameters()) + list(hd.parameters())
        tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask),
                          grad_sync=GradSync(params, mode=mode, bucket_mb=1.0))
        opt = torch.optim.SGD(params, lr=0.0)
        tr.grad_sync.begin_step()
        _, _, loss = tr.forward_loss(batch, L.rmse_mse_padded_loss)
        loss.backward()
        tr.grad_sync.finish()
        grads[mode] = [p.grad.detach().clone() for p in params]
    err = max((a - b).abs().max().item() / (b.abs().max().item() + 1e-12)
              for a, b in zip(grads["fused"], grads["nccl"]) if b.numel())
    return err


def test_fused_grad_sync_matches_nccl_in_training():
    _need(2)
    out = _dist_util.run(_train_worker, world=2, backend="nccl")
    assert max(out.values()) < 1e-5, out
