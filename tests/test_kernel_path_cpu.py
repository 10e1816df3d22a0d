"""The whole kernel path of the model (every op the training step sends to the extension) run
on the CPU through a stand-in for the extension (``tests/cpu_extension.py``) and compared with
the PyTorch path: forward outputs, loss and every parameter gradient.  This checks the Python
side of the kernel path - buffer layouts, views and strides handed to the kernels, GEMM problem
grouping, padding, the autograd functions - without a GPU."""
import numpy as np
import pytest
import torch

from tests.cpu_extension import use_cpu_extension


def _model(mmax, message_type="source-target", **extra):
    from maloq_b200.data import basis_sets, structures
    from maloq_b200.data.batch import collate, make_sample
    from maloq_b200.data.targets import FockLabeler
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head

    lab = FockLabeler(basis_sets.get_basis("split_valence_small"))
    rng = np.random.default_rng(4)
    samples = [make_sample(structures.random_small_molecule(rng), 5.0) for _ in range(3)]
    torch.manual_seed(11)
    for s in samples:
        s.node_y = torch.randn(1, s.num_nodes, lab.target_len)
        s.y = torch.randn(1, s.num_edges, lab.target_len)
    b = collate(samples, lab.table)
    torch.manual_seed(0)
    kw = dict(sphere_channels=16, hidden_channels=16, lmax=4, mmax=mmax, cutoff=5.0, num_layers=2,
              num_distance_basis=8, edge_channels=16, message_type=message_type, **extra)
    bb = eSEN_Backbone(lab.irreps, include_edges=True, **kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=16, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True)
    return bb, hd, b, lab


def _step(bb, hd, b, lab):
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask))
    for p in list(bb.parameters()) + list(hd.parameters()):
        p.grad = None
    ln, le, loss = tr.forward_loss(b, L.rmse_mse_padded_loss)
    loss.backward()
    grads = {n: p.grad.clone() for n, p in list(bb.named_parameters()) + [("head." + k, v) for k, v in hd.named_parameters()]
             if p.grad is not None}
    return float(ln.detach()), float(le.detach()), float(loss.detach()), grads


@pytest.mark.parametrize("mmax,message_type", [(2, "source-target"), (2, "source-target-message"),
                                               (4, "source-target"), (1, "source-target")])
def test_kernel_path_matches_pytorch_path_on_cpu(monkeypatch, mmax, message_type):
    bb, hd, b, lab = _model(mmax, message_type)
    ref = _step(bb, hd, b, lab)
    ext = use_cpu_extension(monkeypatch)
    got = _step(bb, hd, b, lab)
    expected = {"gemm", "edge_rotation", "gather_rotate_fwd", "gather_rotate_bwd", "gate_fwd",
                "gate_bwd", "rotate_back_scatter", "rotate_back_edge", "rotate_grad", "rms_norm_fwd", "rms_norm_bwd",
                "ln_silu_fwd", "ln_silu_bwd", "gate_l_fwd", "gate_l_bwd", "head_gate_fwd", "head_gate_bwd",
                "fock_loss_stats", "fock_loss_grad"}
    assert expected <= set(ext.calls), expected - set(ext.calls)
    for a, r in zip(got[:3], ref[:3]):
        assert abs(a - r) <= 3e-2 * abs(r), (a, r)
    assert set(got[3]) == set(ref[3])
    worst = []
    for n, g in ref[3].items():
        d = (got[3][n] - g).norm() / (g.norm() + 1e-12)
        worst.append((float(d), n))
    worst.sort(reverse=True)
    assert worst[0][0] < 5e-2, worst[:5]


@pytest.mark.parametrize("extra", [dict(edge_chunk=40, edge_stream_dtype=torch.float32), dict(edge_chunk=40),
                                   dict(activation_checkpointing=True)])
def test_chunked_and_recomputed_kernel_paths_match_on_cpu(monkeypatch, extra):
    """Edge-chunked execution (per-chunk recompute, fp32 or bf16 edge stream) and block
    recompute on the kernel path against the unchunked PyTorch path."""
    bb, hd, b, lab = _model(2)
    ref = _step(bb, hd, b, lab)
    bb2, hd2, _, _ = _model(2, **extra)
    bb2.load_state_dict(bb.state_dict())
    hd2.load_state_dict(hd.state_dict())
    ext = use_cpu_extension(monkeypatch)
    got = _step(bb2, hd2, b, lab)
    assert ext.calls.get("gather_rotate_fwd", 0) > 0
    tol = 2e-2 if extra.get("edge_stream_dtype", torch.bfloat16) == torch.float32 or "edge_chunk" not in extra else 4e-2
    for a, r in zip(got[:3], ref[:3]):
        assert abs(a - r) <= tol * abs(r), (a, r)
    worst = max(float((got[3][n] - g).norm() / (g.norm() + 1e-12)) for n, g in ref[3].items())
    assert worst < 2.5 * tol, worst


def _train_mae(steps, kernel_path, monkeypatch):
    """Train the small model on fixed synthetic Fock targets; Hamiltonian MAE of the result."""
    from maloq_b200.data import datasets
    from maloq_b200.data.batch import collate
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    lab = datasets.labeler_for("small")
    kw = dict(sphere_channels=16, hidden_channels=16, lmax=4, mmax=2, cutoff=5.0, num_layers=2,
              num_distance_basis=8, edge_channels=16)
    samples, _ = datasets.build_dataset("small", 6, kw, seed=3, labeler=lab)
    b = collate(samples, lab.table)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, include_edges=True, **kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=16, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True)
    if kernel_path:
        use_cpu_extension(monkeypatch)
    opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()), lr=3e-3)
    tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask))
    for _ in range(steps):
        tr.train_step(b, L.rmse_mse_padded_loss, opt)
    with torch.no_grad():
        no, eo = hd(bb(b), b)
    maes = []
    n0 = e0 = 0
    for s in samples:  # per molecule: predicted vs target Hamiltonian blocks
        n1, e1 = n0 + s.num_nodes, e0 + s.num_edges
        Hp = lab.blocks_from_labels(s, no[0][n0:n1], eo[0][e0:e1]).to_dense()
        Ht = lab.blocks_from_labels(s, s.node_y[0], s.y[0]).to_dense()
        maes.append(float(np.abs(Hp - Ht).mean()))
        n0, e0 = n1, e1
    return float(np.mean(maes))


def test_trained_hamiltonian_mae_matches_pytorch_path(monkeypatch):
    """Hamiltonian MAE after the same training run on the PyTorch path (fp32) and on the kernel
    path (bf16 GEMM operands, CPU stand-in): the reduced-precision operands do not cost
    accuracy at this scale (within 10 %), and both improve on the untrained model."""
    mae0 = _train_mae(0, False, monkeypatch)
    ref = _train_mae(40, False, monkeypatch)
    got = _train_mae(40, True, monkeypatch)
    assert ref < 0.7 * mae0 and got < 0.7 * mae0, (mae0, ref, got)
    assert abs(got - ref) <= 0.1 * ref, (ref, got)


@pytest.mark.parametrize("extra", [{}, dict(edge_chunk=40), dict(edge_chunk=40, edge_stream_dtype=torch.float32),
                                   dict(activation_checkpointing=True)])
def test_kernel_path_reads_no_uninitialised_memory(monkeypatch, extra):
    """With PyTorch filling every new uninitialised tensor with NaN, one training step on the
    kernel path (CPU stand-in) stays finite: no buffer handed to a kernel is read before it is
    written."""
    import torch.utils.deterministic as det

    bb, hd, b, lab = _model(2, "source-target-message", **extra)
    old_mode, old_fill = torch.are_deterministic_algorithms_enabled(), det.fill_uninitialized_memory
    torch.use_deterministic_algorithms(True, warn_only=True)
    det.fill_uninitialized_memory = True
    try:
        use_cpu_extension(monkeypatch)
        ln, le, loss, grads = _step(bb, hd, b, lab)
    finally:
        torch.use_deterministic_algorithms(old_mode)
        det.fill_uninitialized_memory = old_fill
    assert np.isfinite([ln, le, loss]).all()
    bad = [n for n, g in grads.items() if not torch.isfinite(g).all()]
    assert not bad, bad


@pytest.mark.parametrize("kind", ["energies", "forces"])
def test_energy_and_force_heads_on_the_kernel_path(monkeypatch, kind):
    """Energy / force heads (an extra Edgewise convolution on the node embeddings) on the kernel
    path against the PyTorch path: loss and gradients."""
    from maloq_b200.models.heads import HELM_Energy_Head, HELM_Force_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    bb, _, b, lab = _model(2)
    torch.manual_seed(2)
    hd = (HELM_Energy_Head if kind == "energies" else HELM_Force_Head)(bb)
    # zero targets: the loss is the mean square of the prediction, so its relative error is the
    # prediction's (random targets can cancel most of a prediction and magnify its error)
    if kind == "energies":
        b.energy = torch.zeros(b.num_graphs)
    else:
        b.forces = torch.zeros(b.num_nodes, 3)

    def step():
        tr = SplitTrainer(bb, hd, lab.irreps)
        for p in list(bb.parameters()) + list(hd.parameters()):
            p.grad = None
        _, _, loss = tr.forward_loss(b, L.mse_padded_loss)
        loss.backward()
        return float(loss.detach()), {n: p.grad.clone() for n, p in hd.named_parameters() if p.grad is not None}

    ref = step()
    use_cpu_extension(monkeypatch)
    got = step()
    assert abs(got[0] - ref[0]) <= 2e-2 * abs(ref[0])
    for n, g in ref[1].items():
        assert ((got[1][n] - g).norm() / (g.norm() + 1e-12)).item() < 5e-2, n


@pytest.mark.parametrize("head_kw", [dict(open_shell=True), dict(reduce_edge=True), dict(reduce_node=False),
                                     dict(reduce_node=True, reduce_node_intra=False)])
def test_fock_head_variants_on_the_kernel_path(monkeypatch, head_kw):
    """Open-shell (two spin channels), reduce_edge (tanh gates of |u|, half-edge pairs) and the
    node-reduction variants of the Fock head on the kernel path against the PyTorch path."""
    from maloq_b200.models.heads import Fock_Irreps_Head

    bb, _, b, lab = _model(2)
    torch.manual_seed(3)
    kw = dict(reduce_node=True, reduce_node_intra=True)
    kw.update(head_kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=16, ls_list=lab.layout.ls_list, **kw)
    if head_kw.get("open_shell"):
        b.node_y = torch.cat([b.node_y, b.node_y * 0.5])
        b.y = torch.cat([b.y, b.y * 0.5])

    def step():
        for p in list(bb.parameters()) + list(hd.parameters()):
            p.grad = None
        no, eo = hd(bb(b), b)
        g1, g2 = torch.randn_like(no, generator=torch.Generator().manual_seed(1)), \
            torch.randn_like(eo, generator=torch.Generator().manual_seed(2))
        ((no * g1).sum() + (eo * g2).sum()).backward()
        return no.detach(), eo.detach(), {n: p.grad.clone() for n, p in hd.named_parameters() if p.grad is not None}

    ref = step()
    use_cpu_extension(monkeypatch)
    got = step()
    rel = lambda a, r: ((a - r).norm() / (r.norm() + 1e-12)).item()
    assert got[0].shape == ref[0].shape and got[1].shape == ref[1].shape
    assert rel(got[0], ref[0]) < 2e-2 and rel(got[1], ref[1]) < 2e-2
    for n, g in ref[2].items():
        assert rel(got[2][n], g) < 5e-2, n


@pytest.mark.parametrize("norm_type", ["layer_norm", "layer_norm_sh"])
def test_norm_variants_on_the_kernel_path(monkeypatch, norm_type):
    """The layer-norm variants (PyTorch ops) inside blocks whose other ops run on the kernel path."""
    bb, hd, b, lab = _model(2, norm_type=norm_type)
    ref = _step(bb, hd, b, lab)
    use_cpu_extension(monkeypatch)
    got = _step(bb, hd, b, lab)
    assert abs(got[2] - ref[2]) <= 2e-2 * abs(ref[2])
    worst = max(float((got[3][n] - g).norm() / (g.norm() + 1e-12)) for n, g in ref[3].items())
    assert worst < 5e-2, worst


@pytest.mark.parametrize("target", ["fock_matrix", "forces"])
def test_workflow_trains_on_the_kernel_path(monkeypatch, tmp_path, target):
    """The training workflow (data, trainer, optimizer step with the bf16 weight cache,
    checkpoints) on the kernel path: the loss falls over a few epochs."""
    from maloq.train_utils import training_workflow

    use_cpu_extension(monkeypatch)
    cfg = dict(dataset_name="synthetic_small", num_structures=8, batch_size=4, num_epochs=4, l_embedding_dim=16,
               num_mp_layers=1, num_distance_basis=8, rcut_orbitals=2.5, rcut_gaussian=5.0, mmax=2, lr_init=3e-3,
               output_folder=str(tmp_path), device="cpu", log_every=0, loss_target=target)
    hist = training_workflow.TrainingWorkflow(cfg).run()
    tr = hist["train_node"] if target == "fock_matrix" else [a + b for a, b in zip(hist["train_node"],
                                                                                   hist["train_edge"])]
    assert np.isfinite(tr).all() and tr[-1] < tr[0], tr


def test_lmax6_frame_on_the_kernel_path(monkeypatch):
    """The lmax 6 / mmax 2 frame of the large-molecule configuration (def2-TZVP-like basis, f
    shells) on the kernel path against the PyTorch path."""
    from maloq_b200.data import datasets
    from maloq_b200.data.batch import collate
    from maloq_b200.models.backbone import eSEN_Backbone
    from maloq_b200.models.heads import Fock_Irreps_Head

    lab = datasets.labeler_for("large")
    assert lab.layout.lmax == 6
    samples = datasets.build_samples("large", 1, seed=2)
    samples = [s for s in samples]
    torch.manual_seed(5)
    for s in samples:
        s.node_y = torch.randn(1, s.num_nodes, lab.target_len)
        s.y = torch.randn(1, s.num_edges, lab.target_len)
    b = collate(samples, lab.table)
    kw = dict(sphere_channels=8, hidden_channels=8, lmax=6, mmax=2, cutoff=6.0, num_layers=1, num_distance_basis=8,
              edge_channels=8)
    torch.manual_seed(0)
    bb = eSEN_Backbone(lab.irreps, include_edges=True, **kw)
    hd = Fock_Irreps_Head(None, lab.irreps, lmax=6, sphere_channels=8, ls_list=lab.layout.ls_list,
                          reduce_node=True, reduce_node_intra=True)
    ref = _step(bb, hd, b, lab)
    use_cpu_extension(monkeypatch)
    got = _step(bb, hd, b, lab)
    assert abs(got[2] - ref[2]) <= 3e-2 * abs(ref[2])
    errs = sorted(float((got[3][n] - g).norm() / (g.norm() + 1e-12)) for n, g in ref[3].items())
    # 8 channels: bf16 operand noise is larger than at production widths
    assert errs[-1] < 8e-2 and errs[len(errs) // 2] < 2e-2, errs[-5:]


def test_streamed_inference_on_the_kernel_path(monkeypatch):
    """Chunked, gradient-free inference on the kernel path (edge stream overwritten in place,
    rotations computed per chunk, bf16 stream) and the streamed block-sparse Hamiltonian shard,
    against the unchunked PyTorch path."""
    from maloq_b200.parallel.infer import hamiltonian_shard

    bb, hd, b, lab = _model(2)
    tbl = lab.table
    b.edge_pair_type = torch.as_tensor(tbl.pair_type(b.src_z.numpy(), b.dst_z.numpy()))
    b.node_pair_type = torch.as_tensor(tbl.pair_type(b.atomic_numbers.numpy(), b.atomic_numbers.numpy()))
    with torch.no_grad():
        emb = bb(b)
        no, eo = hd(emb, b)
        ref_data, ref_ptr = hamiltonian_shard(hd, emb, b, lab)
    bb2, hd2, _, _ = _model(2, edge_chunk=30)
    bb2.load_state_dict(bb.state_dict())
    hd2.load_state_dict(hd.state_dict())
    ext = use_cpu_extension(monkeypatch)
    with torch.no_grad():
        g = bb2.build_graph(b)
        assert g.rot is None and len(g.chunks) > 1
        emb2 = bb2(b)
        no2, eo2 = hd2(emb2, b)
        data, ptr = hamiltonian_shard(hd2, emb2, b, lab)
    assert ext.calls.get("gather_rotate_fwd", 0) > 0 and ext.calls.get("basis_rows", 0) > 0
    rel = lambda a, r: ((a.double() - r.double()).norm() / r.double().norm()).item()
    assert rel(no2, no) < 2e-2 and rel(eo2, eo) < 3e-2
    assert torch.equal(ptr, ref_ptr) and rel(data, ref_data) < 3e-2


def test_driver_smoke_on_the_cpu_stand_in(monkeypatch):
    """The driver's smoke() (tiny flagship forward + backward: teacher targets, label rows,
    model, fused loss) on the kernel path through the CPU stand-in."""
    import __graft_entry__ as entry

    ext = use_cpu_extension(monkeypatch)
    entry.smoke("cpu")
    assert {"gather_rotate_fwd", "head_gate_fwd", "basis_rows", "fock_loss_stats", "gather_rotate_bwd"} <= set(ext.calls)


_SYNC_OPS = {"_local_scalar_dense", "nonzero", "masked_select", "lift_fresh", "lift_fresh_copy", "repeat_interleave",
             "unique", "_unique2", "bincount"}


def _sync_census(step):
    """ATen ops of ``step`` that would make the host wait for the device (reading a value back,
    data-dependent output sizes) or copy host data to it, excluding ops of the CPU stand-in."""
    import traceback

    from torch.utils._python_dispatch import TorchDispatchMode

    class Census(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.hits = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            name = func.overloadpacket.__name__
            masked = name in ("index", "index_put", "index_put_") and any(
                isinstance(t, torch.Tensor) and t.dtype == torch.bool for t in (args[1] if len(args) > 1 else []))
            if name in _SYNC_OPS or masked:  # boolean-mask indexing has a data-dependent size
                st = traceback.extract_stack()
                # the stand-in's own ops, and torch.optim's step counters (host tensors on a GPU too)
                if not any("cpu_extension.py" in f.filename or "fake_symm.py" in f.filename or
                           "torch/optim" in f.filename for f in st):
                    site = [f"{f.filename.split('repo/')[-1]}:{f.lineno}" for f in st if "maloq_b200" in f.filename]
                    self.hits.append((name, site[-1] if site else "?"))
            return func(*args, **(kwargs or {}))

    c = Census()
    with c:
        step()
    return c.hits


@pytest.mark.parametrize("head_kw,extra", [({}, {}), (dict(reduce_edge=True), {}), ({}, dict(edge_chunk=40))])
def test_training_step_has_no_host_synchronisation(monkeypatch, head_kw, extra):
    """A steady-state training step (forward, fused loss, backward, optimizer step with the bf16
    weight-cache refresh) on the kernel path issues no op that would stall the host on a GPU:
    no value read back, no data-dependent output size, no host data copied to the device."""
    from maloq_b200.models.heads import Fock_Irreps_Head
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    bb, hd, b, lab = _model(2, **extra)
    if head_kw:
        hd = Fock_Irreps_Head(None, lab.irreps, lmax=4, sphere_channels=16, ls_list=lab.layout.ls_list,
                              reduce_node=True, **head_kw)
    use_cpu_extension(monkeypatch)
    opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()), lr=1e-3)
    tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask))
    tr.train_step(b, L.rmse_mse_padded_loss, opt)  # first step: caches and tables are built
    hits = _sync_census(lambda: tr.train_step(b, L.rmse_mse_padded_loss, opt))
    assert not hits, hits
    # the census does see such ops when they come from the package
    from maloq_b200.ops import reference as R

    assert _sync_census(lambda: R.fock_loss(torch.ones(2, 3), torch.ones(2, 3), torch.zeros(2, 3), torch.zeros(2, 3),
                                            torch.ones(2, 3, dtype=torch.bool), torch.ones(2, 3, dtype=torch.bool),
                                            L.mse_padded_loss))


def _op_census(step):
    """(op name, last package frame) -> count of the ATen ops of ``step`` outside the CPU stand-in
    and torch.optim, views and allocations excluded: on a GPU each is a launch of its own."""
    import collections
    import traceback

    from torch.utils._python_dispatch import TorchDispatchMode

    free = {"view", "_unsafe_view", "slice", "select", "as_strided", "t", "transpose", "detach", "alias", "unsqueeze",
            "squeeze", "expand", "permute", "reshape", "split", "split_with_sizes", "unbind", "narrow", "empty",
            "empty_like", "empty_strided", "new_empty", "new_empty_strided", "is_same_size"}
    cnt = collections.Counter()

    class Census(TorchDispatchMode):
        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            name = func.overloadpacket.__name__
            if name not in free:
                st = traceback.extract_stack()
                if not any("cpu_extension.py" in f.filename or "torch/optim" in f.filename for f in st):
                    site = [f"{f.filename.split('repo/')[-1]}:{f.lineno}" for f in st if "maloq_b200" in f.filename]
                    cnt[(name, site[-1] if site else "?")] += 1
            return func(*args, **(kwargs or {}))

    with Census():
        step()
    return cnt


def test_training_step_launch_budget(monkeypatch):
    """Glue ops of a steady-state training step stay few: column sums (bias gradients, norm
    partials, per-degree weight-gradient sums) run in the extension, the optimizer step rewrites
    the whole bf16 weight cache through the extension, and the total stays within a budget."""
    from maloq_b200.ops import weights as W
    from maloq_b200.train import loss as L
    from maloq_b200.train.trainer import SplitTrainer

    bb, hd, b, lab = _model(2)
    ext = use_cpu_extension(monkeypatch)
    W.invalidate()
    opt = torch.optim.Adam(list(bb.parameters()) + list(hd.parameters()), lr=1e-3)
    tr = SplitTrainer(bb, hd, lab.irreps, mask_table=torch.as_tensor(lab.table.mask))
    tr.train_step(b, L.rmse_mse_padded_loss, opt)
    packs = ext.calls.get("weight_pack", 0)
    cnt = _op_census(lambda: tr.train_step(b, L.rmse_mse_padded_loss, opt))
    sums = {k: v for k, v in cnt.items() if k[0] == "sum" and k[1].startswith("maloq_b200/ops/")}
    assert not sums, sums
    from_cache = sum(v for k, v in cnt.items() if k[1].startswith("maloq_b200/ops/weights.py"))
    assert from_cache <= 6, from_cache  # only non-parameter weights (padded head views) are cast per call
    assert ext.calls["weight_pack"] > packs
    assert sum(cnt.values()) <= 320, sorted(cnt.items(), key=lambda kv: -kv[1])[:20]
    W.invalidate()
