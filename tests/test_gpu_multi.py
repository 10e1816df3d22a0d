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


@pytest.mark.parametrize("multimem", [False, True])
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


def _partition_worker(rank, world, transport, edge_chunk=None):
    import numpy as np
    import torch

    from maloq_b200.data import batch as B
    from maloq_b200.data import basis_sets, structures
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.ops import kernels
    from maloq_b200.parallel import partition as P
    from maloq_b200.parallel.halo import partition_batch

    dev = torch.device("cuda", rank)
    rng = np.random.default_rng(0)
    s = structures.Structure(rng.choice([1, 6, 8], size=300), rng.uniform(0, 16, size=(300, 3)))
    g = B.make_sample(s, 5.0)
    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    kw = dict(sphere_channels=32, hidden_channels=32, lmax=4, mmax=2, cutoff=5.0, num_layers=2, num_distance_basis=16,
              edge_channels=32)

    def model(chunk=None):
        torch.manual_seed(0)
        bb = eSEN_Backbone(lab.irreps, edge_chunk=chunk, edge_stream_dtype=torch.float32, **kw).to(dev)
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=32, ls_list=lab.layout.ls_list,
                              reduce_node=True, reduce_node_intra=True).to(dev)
        return bb, hd

    def run(batch, own, edges, chunk=None):
        bb, hd = model(chunk)
        no, eo = hd(bb(batch), batch)
        torch.manual_seed(7)
        wn = torch.randn(g.num_nodes, no.shape[-1], device=dev)
        we = torch.randn(len(g.src), eo.shape[-1], device=dev)
        loss = (no[0] * wn[own]).sum() + (eo[0] * we[edges]).sum()
        loss.backward()
        named = [(n, p) for n, p in list(bb.named_parameters()) + [("head." + k, v) for k, v in hd.named_parameters()]]
        return no[0].detach(), eo[0].detach(), named

    # unpartitioned reference on this GPU
    full = B.collate([g], lab.table).to(dev)
    _, _, ref_named = run(full, torch.arange(g.num_nodes, device=dev), torch.arange(len(g.src), device=dev))
    part = P.partition("rcb", g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    dom = P.decompose(part, g.src, g.dst, world)[rank]
    b = partition_batch(g, dom, lab.table, device=dev, transport=transport)
    no, eo, named = run(b, torch.as_tensor(dom.owned, device=dev), torch.as_tensor(dom.edges, device=dev), edge_chunk)
    errs = {}
    for (n, p), (_, rp) in zip(named, ref_named):
        if p.numel() == 0:
            continue
        gr = p.grad if p.grad is not None else torch.zeros_like(p)
        torch.distributed.all_reduce(gr)
        rg = rp.grad if rp.grad is not None else torch.zeros_like(rp)
        errs[n] = ((gr - rg).abs().max() / (rg.abs().max() + 1e-6)).item()
    torch.cuda.synchronize()
    return no.cpu(), eo.cpu(), errs, kernels.error_status()


@pytest.mark.parametrize("transport,edge_chunk", [("collective", None), ("peer", None), ("peer", 1500),
                                                  ("collective", 1500)])
def test_partitioned_gpu_matches_unpartitioned(transport, edge_chunk):
    """2 GPUs, graph-partitioned = unpartitioned; the in-kernel peer halo, and with
    ``edge_chunk`` the chunked blocks sharing one halo exchange (peer fetch) per block."""
    _need(2)
    out = _dist_util.run(_partition_worker, world=2, backend="nccl", args=(transport, edge_chunk))
    for r in range(2):
        _, _, errs, status = out[r]
        assert status == 0
        bad = {k: v for k, v in errs.items() if v > 2e-2}
        assert not bad, (transport, bad)
