"""Failure detection on the host (gloo ranks): a rank that raises, a rank that never joins, a
delayed rank, a corrupted halo plan, mismatched batch counts, a non-finite loss.  No GPU is
faulted, trapped or hung."""
import datetime

import pytest
import torch

from tests import _dist_util


def _raising_worker(rank, world):
    import torch.distributed as dist

    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    dist.barrier()
    return "unreachable"


def test_raising_rank_is_reported():
    with pytest.raises(AssertionError, match="injected failure"):
        _dist_util.run(_raising_worker, world=2, timeout=60)


def test_missing_rank_times_out():
    import torch.distributed as dist

    store = dist.TCPStore("127.0.0.1", _dist_util.free_port(), 2, True, timeout=datetime.timedelta(seconds=2),
                          wait_for_workers=False)
    with pytest.raises(Exception):
        dist.init_process_group("gloo", store=store, rank=0, world_size=2, timeout=datetime.timedelta(seconds=2))
    if dist.is_initialized():
        dist.destroy_process_group()


def _batch_mismatch_worker(rank, world):
    from maloq_b200.train.trainer import SplitTrainer

    tr = SplitTrainer(torch.nn.Linear(1, 1), torch.nn.Linear(1, 1), None)
    try:
        tr.check_batch_consistency(3 + rank, 2, "cpu")
    except ValueError as e:
        return str(e)
    return "no error"


def test_batch_count_mismatch_detected():
    out = _dist_util.run(_batch_mismatch_worker, world=2)
    assert all("Mismatch" in v for v in out.values())


def test_nan_guard_stops_step():
    import numpy as np

    from maloq_b200.data import basis_sets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    s = make_sample(structures.random_small_molecule(np.random.default_rng(0)), 5.0)
    n, e = s.num_nodes, s.num_edges
    s.node_y = torch.zeros(1, n, lab.target_len)
    s.y = torch.zeros(1, e, lab.target_len)
    s.y[0, 0, 0] = float("nan")  # corrupted target
    b = collate([s], lab.table)
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=4, mmax=2, cutoff=5.0, num_layers=1, num_distance_basis=8,
              edge_channels=8)
    bb = eSEN_Backbone(lab.irreps, **kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=8, ls_list=lab.layout.ls_list)
    tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.ones(lab.table.mask.shape, dtype=torch.bool),
                      nan_guard=True)
    opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()))
    before = [p.detach().clone() for p in bb.parameters()]
    with pytest.raises(FloatingPointError):
        tr.train_step(b, L.mse_padded_loss, opt)
    assert all(torch.equal(a, p) for a, p in zip(before, bb.parameters()))


def _plan_worker(rank, world, corrupt):
    from maloq_b200.parallel import partition as P
    from maloq_b200.parallel.halo import HaloPlan, HaloPlanError
    from tests.test_partition_cpu import _toy_graph

    g = _toy_graph()
    part = P.partition("slab", g.num_nodes, world, src=g.src, dst=g.dst, pos=g.pos)
    dom = P.decompose(part, g.src, g.dst, world)[rank]
    if corrupt and rank == 1:  # a stale plan: one row fewer sent to rank 0
        dom.send[0] = dom.send[0][:-1]
    try:
        HaloPlan(dom, "cpu")
    except HaloPlanError as e:
        return str(e)
    return "ok"


@pytest.mark.parametrize("corrupt", [False, True])
def test_corrupted_halo_plan_is_detected_on_every_rank(corrupt):
    out = _dist_util.run(_plan_worker, world=2, args=(corrupt,))
    if corrupt:
        assert all("inconsistent halo plans" in v and "rank 0 expects" in v for v in out.values())
    else:
        assert all(v == "ok" for v in out.values())


def _slow_worker(rank, world):
    import time

    import torch.distributed as dist

    if rank == 1:
        time.sleep(3.0)  # a straggler: late, but within the process-group timeout
    t = torch.ones(4) * (rank + 1)
    dist.all_reduce(t)
    return float(t[0])


def test_delayed_rank_completes_within_timeout():
    out = _dist_util.run(_slow_worker, world=2)
    assert all(v == 3.0 for v in out.values())


def _crash_resume_worker(rank, world, folder, phase):
    """phase "full": 3 epochs uninterrupted; "crash": rank 1 raises in its first step of epoch 3
    (after the epoch-2 checkpoint); "resume": restart from the checkpoint and finish epoch 3."""
    from maloq_b200.train import trainer as T
    from maloq.train_utils import training_workflow

    cfg = dict(dataset_name="synthetic_small", num_structures=12, num_val=2, batch_size=3, num_epochs=3,
               l_embedding_dim=8, num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0,
               mmax=2, output_folder=folder, device="cpu", save_frequency=1, log_every=0, lr_init=3e-3)
    if phase == "resume":
        cfg.update(restart_backbone=True, restart_head=True, restart_optimizer=True)
    if phase == "crash" and rank == 1:
        step = T.SplitTrainer.train_step
        calls = [0]

        def failing_step(self, *a, **k):
            calls[0] += 1
            if calls[0] == 2 * 2 + 1:  # two batches per epoch on each rank
                raise RuntimeError("injected crash on rank 1")
            return step(self, *a, **k)

        T.SplitTrainer.train_step = failing_step
    try:
        hist = training_workflow.TrainingWorkflow(cfg).run()
    except Exception as e:  # noqa: BLE001 - the failure is the result of this phase
        return "crashed: " + type(e).__name__ + ": " + str(e)[:200]
    sd = torch.load(f"{folder}/backbone.pt", weights_only=False)["model_state_dict"]
    return hist["train_node"], {k: v for k, v in sd.items() if v.is_floating_point()}


def test_crashed_rank_ends_the_job_and_resume_matches_uninterrupted_run(tmp_path):
    """A rank that raises mid-training ends the job on every rank (the other rank's collective
    fails instead of hanging); restarting from the last checkpoint (weights, optimizer,
    scheduler, epoch, RNG) reproduces the uninterrupted run bit for bit."""
    full = _dist_util.run(_crash_resume_worker, world=2, args=(str(tmp_path / "full"), "full"))
    crash = _dist_util.run(_crash_resume_worker, world=2, args=(str(tmp_path / "run"), "crash"), timeout=300)
    assert "injected crash" in crash[1]
    assert crash[0].startswith("crashed")
    res = _dist_util.run(_crash_resume_worker, world=2, args=(str(tmp_path / "run"), "resume"))
    h_full, sd_full = full[0]
    h_res, sd_res = res[0]
    assert len(h_res) == 3 and h_res == h_full
    for k in sd_full:
        assert (sd_full[k] == sd_res[k]).all(), k


def _missing_peer_worker(rank, world, folder):
    import torch.distributed as dist

    from tests import fake_symm
    from tests.cpu_extension import CpuExtension

    symm = fake_symm.install(folder)
    lib = CpuExtension(barrier_timeout=1.0)
    buf = symm.empty(64)
    hdl = symm.rendezvous(buf)
    pads = torch.tensor(hdl.signal_pad_ptrs, dtype=torch.int64)
    lib.peer_barrier(pads.data_ptr(), rank, world, 1, 0, 0)  # everyone arrives
    first = lib.error_status(True)
    if rank == 1:  # rank 1 leaves between steps: it never reaches the second barrier
        dist.barrier()
        return first, None
    lib.peer_barrier(pads.data_ptr(), rank, world, 2, 0, 0)
    second = lib.error_status(True)
    dist.barrier()
    return first, second


def test_missing_peer_at_a_peer_barrier_is_reported(tmp_path):
    """A rank that stops before a peer barrier: the other rank's bounded wait gives up and
    records the peer-wait error (code 4) instead of hanging; the barrier that everyone reached
    records nothing.  Peer memory is emulated in shared memory across gloo processes."""
    out = _dist_util.run(_missing_peer_worker, world=2, args=(str(tmp_path),), timeout=120)
    assert out[0] == (0, 4)
    assert out[1][0] == 0
