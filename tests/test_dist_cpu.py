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
