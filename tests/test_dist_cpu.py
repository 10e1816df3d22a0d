"""Multi-process (gloo, CPU) tests of the data-parallel gradient synchronisation."""
import torch

from tests import _dist_util


def _grad_sync_worker(rank, world, mode):
    import torch

    from maloq_b200.parallel.dp import GradSync

    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.SiLU(), torch.nn.Linear(32, 8))
    sync = GradSync(list(model.parameters()), bucket_mb=0.001, mode=mode)
    outs = []
    for step in range(2):
        torch.manual_seed(100 + 10 * step + rank)
        x = torch.randn(5, 16)
        sync.begin_step()
        model(x).square().sum().backward()
        sync.finish()
        outs.append([p.grad.clone() for p in model.parameters()])
        for p in model.parameters():
            p.grad = None
    return outs


def _expected(world):
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.SiLU(), torch.nn.Linear(32, 8))
    out = []
    for step in range(2):
        acc = [torch.zeros_like(p) for p in model.parameters()]
        for r in range(world):
            torch.manual_seed(100 + 10 * step + r)
            x = torch.randn(5, 16)
            model.zero_grad()
            model(x).square().sum().backward()
            for a, p in zip(acc, model.parameters()):
                a += p.grad / world
        out.append(acc)
    return out


def test_grad_sync_bucketed_matches_average():
    res = _dist_util.run(_grad_sync_worker, world=2, args=("nccl",))  # "nccl" mode = async collective per bucket
    exp = _expected(2)
    for r in range(2):
        for got_step, exp_step in zip(res[r], exp):
            for g, e in zip(got_step, exp_step):
                assert torch.allclose(torch.as_tensor(g), e, atol=1e-6)


def test_grad_sync_per_param_matches_average():
    res = _dist_util.run(_grad_sync_worker, world=2, args=("per_param",))
    exp = _expected(2)
    for got_step, exp_step in zip(res[0], exp):
        for g, e in zip(got_step, exp_step):
            assert torch.allclose(torch.as_tensor(g), e, atol=1e-6)


def _fused_worker(rank, world, folder):
    from maloq_b200.ops import kernels
    from tests import fake_symm
    from tests.cpu_extension import CpuExtension

    fake_symm.install(folder)
    kernels._lib = CpuExtension()
    out = _grad_sync_worker(rank, world, "fused")
    return out, kernels._lib.error_status(True)


def test_fused_allreduce_on_emulated_peer_memory(tmp_path):
    """The fused gradient all-reduce (buckets in one symmetric buffer, a peer barrier per bucket,
    each rank reducing its chunk over every rank's buffer and writing it back, a closing barrier)
    on symmetric memory emulated in shared memory across gloo processes: every rank's gradients
    equal the average over ranks, at 2 and 3 ranks (uneven chunks)."""
    for world in (2, 3):
        out = _dist_util.run(_fused_worker, world=world, args=(str(tmp_path / f"w{world}"),), timeout=300)
        exp = _expected(world)
        for r, (steps, err) in out.items():
            assert err == 0
            for got, ref in zip(steps, exp):
                for a, b in zip(got, ref):
                    assert torch.allclose(torch.as_tensor(a), b, atol=1e-5, rtol=1e-5)
